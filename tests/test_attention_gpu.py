"""GPU parity of the sm_100a kernels (through the C ABI) against the CPU oracle and the
reference's golden vectors.

Bars (the reference's own, runtime/attention.py:40 and the north-star parity): bf16 output
max-abs error <= 2e-2 and per-token cosine >= 0.9999 vs the fp32 CPU path; LSE within 1e-3.
"""

from __future__ import annotations

import pytest
import torch

import oracle
from conftest import golden_names, load_golden, load_rope_golden, packed_inputs, rope_golden_names, rope_tables

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-2
MIN_COS = 0.9999
LSE_ATOL = 1e-3


def _b200():
    import packed_encoders_b200 as pe

    return pe


def _assert_parity(got: torch.Tensor, ref: torch.Tensor, what: str = ""):
    """The north-star bars, unscaled: max-abs <= 2e-2 and per-token cosine >= 0.9999 against the
    fp32 CPU path. Prints the observed errors so parity can be read off the test log."""
    got = got.float().cpu()
    ref = ref.float().cpu()
    assert torch.isfinite(got).all(), f"{what}: non-finite output"
    err = (got - ref).abs().max().item() if got.numel() else 0.0
    cos_min = 1.0
    if got.numel():
        cos = torch.nn.functional.cosine_similarity(got.flatten(1), ref.flatten(1), dim=1)
        cos_min = cos.min().item()
    print(f"PARITY {what}: max_abs={err:.5f} min_cos={cos_min:.7f}")
    assert err <= MAX_ABS, f"{what}: max abs err {err:.3g} > {MAX_ABS}"
    # a zero row (never produced for valid rows) would give cos 0; all rows here are real
    assert cos_min >= MIN_COS, f"{what}: min per-token cosine {cos_min:.6f}"
    return err, cos_min


def _assert_lse(got: torch.Tensor, ref: torch.Tensor, what: str = ""):
    got, ref = got.float().cpu(), ref.float().cpu()
    finite = torch.isfinite(ref)
    assert torch.equal(finite, torch.isfinite(got)), f"{what}: LSE finiteness differs"
    err = (got[finite] - ref[finite]).abs().max().item() if finite.any() else 0.0
    print(f"PARITY {what}: lse_max_abs={err:.6f}")
    assert err <= LSE_ATOL, f"{what}: LSE max abs err {err:.3g} > {LSE_ATOL}"


def _run(q, k, v, cu, *, scale, window=(-1, -1), causal=False, cu_k=None):
    pe = _b200()
    dev = torch.device("cuda")
    lens_q = (cu[1:] - cu[:-1])
    lens_k = lens_q if cu_k is None else (cu_k[1:] - cu_k[:-1])
    out, lse = pe.packed_attention(
        q.to(dev), k.to(dev), v.to(dev), cu.to(dev), int(lens_q.max()) if lens_q.numel() else 0,
        scale=scale, window=window, causal=causal,
        cu_seqlens_k=None if cu_k is None else cu_k.to(dev),
        max_seqlen_k=int(lens_k.max()) if lens_k.numel() else 0, return_lse=True)
    torch.cuda.synchronize()
    assert pe.device_error_word() == 0, f"device error word {pe.device_error_word()}"
    return out, lse


@pytest.mark.parametrize("dim", [64, 128, 256])
def test_layout_probe_qk(dim):
    pe = _b200()
    gen = torch.Generator().manual_seed(dim)
    q = torch.randn(128, dim, generator=gen).to(torch.bfloat16)
    k = torch.randn(100, dim, generator=gen).to(torch.bfloat16)
    s = pe.ops.debug_qk(q.cuda(), k.cuda()).cpu()
    ref = torch.zeros(128, 128)
    ref[:, :100] = q.float() @ k.float().T
    torch.testing.assert_close(s, ref, atol=1e-3, rtol=1e-4)


@pytest.mark.parametrize("dim", [64, 128, 256])
def test_layout_probe_pv(dim):
    pe = _b200()
    gen = torch.Generator().manual_seed(dim + 1)
    p = torch.rand(128, 128, generator=gen)
    v = torch.randn(128, dim, generator=gen).to(torch.bfloat16)
    o = pe.ops.debug_pv(p.cuda(), v.cuda()).cpu()
    ref = p.to(torch.bfloat16).float() @ v.float()
    torch.testing.assert_close(o, ref, atol=1e-3, rtol=1e-4)


# Rounding the EXACT fp32 reference output of this fixture to bf16 already moves it by 0.0221
# (q, k, v scaled by 2 as in tests/test_cpu_short_attention.py:198; |out| reaches 8.1, where half
# a bf16 ulp is 0.031): no bf16 output, however computed, meets 2e-2 absolute on it. Measured on
# B200: this kernel 0.0221, FlashAttention-2 varlen (the reference's compiled-FA path) 0.0221.
# test_golden_vectors_no_worse_than_fa2 checks every fixture, this one included, against FA2.
_BF16_QUANTUM_BOUND = {
    "native_edge_half15": "bf16 rounding of the exact output alone is 0.0221 > 2e-2 (|out| up to 8.1); "
                          "measured: this kernel 0.0221, FA2 varlen 0.0221",
}


def _golden_params():
    return [pytest.param(n, marks=pytest.mark.xfail(strict=True, reason=_BF16_QUANTUM_BOUND[n]))
            if n in _BF16_QUANTUM_BOUND else n for n in golden_names()]


def _run_golden(g):
    return _run(g["q"], g["k"], g["v"], g["cu_q"], scale=g["scale"], window=g["window"], causal=g["causal"],
                cu_k=None if torch.equal(g["cu_q"], g["cu_k"]) else g["cu_k"])


@pytest.mark.parametrize("name", _golden_params())
def test_golden_vectors(name):
    g = load_golden(name)
    out, lse = _run_golden(g)
    _, ref_lse = oracle.attention_prefixed(g["q"], g["k"], g["v"], g["cu_q"], g["cu_k"], scale=g["scale"],
                                           window=g["window"], causal=g["causal"])
    _assert_lse(lse, ref_lse, name)
    _assert_parity(out, g["out"], name)


@pytest.mark.parametrize("name", golden_names())
def test_golden_vectors_no_worse_than_fa2(name):
    """Against the reference's compiled GPU path on the same fixture: FlashAttention-2 varlen
    (packed_encoders/ops.py:364-371; the FA4 build the reference prefers on sm_100 is not in this
    image). Its bf16 output has the same quantum as ours, so its error is the yardstick for the
    fixtures whose exact outputs are too large for a 2e-2 absolute bar."""
    fa = pytest.importorskip("flash_attn")
    g = load_golden(name)
    out, _ = _run_golden(g)
    lq = int((g["cu_q"][1:] - g["cu_q"][:-1]).max())
    lk = int((g["cu_k"][1:] - g["cu_k"][:-1]).max())
    ref_fa = fa.flash_attn_varlen_func(g["q"].cuda(), g["k"].cuda(), g["v"].cuda(), g["cu_q"].cuda(), g["cu_k"].cuda(),
                                       lq, lk, softmax_scale=g["scale"], causal=g["causal"], window_size=g["window"])
    ours = (out.float().cpu() - g["out"]).abs().max().item()
    theirs = (ref_fa.float().cpu() - g["out"]).abs().max().item()
    print(f"PARITY {name}: max_abs={ours:.5f} fa2_max_abs={theirs:.5f}")
    assert ours <= theirs + 1e-3, f"{name}: {ours:.4g} vs FA2 {theirs:.4g}"


CASES = [
    # (lengths, heads, kv_heads, dim, window, causal)
    ([1, 2, 31, 32, 33, 63, 64, 65, 127, 128], 12, 12, 64, (-1, -1), False),
    ([1, 2, 31, 32, 33, 63, 64, 65, 127, 128], 12, 12, 64, (64, 64), False),
    ([128] * 8, 12, 12, 64, (-1, -1), False),
    ([128, 64, 16, 16, 16, 16, 16, 16], 12, 12, 64, (64, 64), False),
    ([46, 46, 45, 45, 45, 44, 43, 42], 12, 12, 64, (-1, -1), False),
    ([300, 129, 1, 2, 513, 77], 4, 4, 64, (-1, -1), False),
    ([300, 129, 1, 2, 513, 77], 4, 4, 64, (64, 64), False),
    ([0, 5, 0, 200, 0], 3, 3, 64, (-1, -1), False),
    ([700, 3, 260], 4, 2, 128, (-1, -1), True),
    ([700, 3, 260], 8, 2, 256, (-1, -1), True),
    ([5, 64, 0, 37, 400], 8, 2, 256, (-1, -1), False),
    ([17, 250, 9], 4, 1, 64, (16, 3), False),
    ([1] * 300 + [129], 2, 2, 64, (-1, -1), False),
]


@pytest.mark.parametrize("lengths,heads,kv_heads,dim,window,causal", CASES)
def test_matches_oracle(lengths, heads, kv_heads, dim, window, causal):
    q, k, v, cu = packed_inputs(lengths, heads, dim, kv_heads=kv_heads, seed=17)
    scale = dim ** -0.5
    out, lse = _run(q, k, v, cu, scale=scale, window=window, causal=causal)
    ref, ref_lse = oracle.attention(q, k, v, cu, scale=scale, window=window, causal=causal)
    what = f"{lengths[:6]} H{heads}/{kv_heads} D{dim} w{window} c{causal}"
    _assert_parity(out, ref, what)
    _assert_lse(lse, ref_lse, what)


@pytest.mark.parametrize("window", [(-1, -1), (64, 64)])
def test_attention_bshd_drop_in(window):
    """ops.attention_bshd's packed form (packed_encoders/ops.py:502-538): [1, T, H, D] views in
    (q, k contiguous from the RoPE pass, v a strided slice of the fused qkv, forward.py:197-205),
    [1, T, H*D] out, against the oracle."""
    pe = _b200()
    lengths, heads = [40, 300, 7, 129, 513], 12
    total = sum(lengths)
    gen = torch.Generator().manual_seed(23)
    qkv = torch.randn(1, total, 3, heads, 64, generator=gen).to(torch.bfloat16)
    cu = torch.tensor([0] + lengths, dtype=torch.int32).cumsum(0, dtype=torch.int32)
    q, k = qkv[:, :, 0].contiguous(), qkv[:, :, 1].contiguous()
    dq, dk, dqkv = q.cuda(), k.cuda(), qkv.cuda()
    out = pe.attention_bshd(dq, dk, dqkv[:, :, 2], window=window, scaling=0.125, cu_seqlens=cu.cuda(),
                            max_seqlen=max(lengths))
    torch.cuda.synchronize()
    assert out.shape == (1, total, heads * 64)
    ref, _ = oracle.attention(q[0], k[0], qkv[0, :, 2], cu, scale=0.125, window=window)
    _assert_parity(out.view(total, heads, 64), ref, f"attention_bshd w{window}")


@pytest.mark.parametrize("window", [(-1, -1), (64, 64)])
def test_flash_attention_varlen_drop_in(window):
    """ops.flash_attention_varlen (packed_encoders/ops.py:432-461): [1, H, T, D] head-major views
    in (the transposed path), [1, T, H*D] out, against the oracle."""
    pe = _b200()
    lengths, heads = [65, 1, 200, 33, 400], 8
    total = sum(lengths)
    gen = torch.Generator().manual_seed(29)
    q, k, v = (torch.randn(1, heads, total, 64, generator=gen).to(torch.bfloat16) for _ in range(3))
    cu = torch.tensor([0] + lengths, dtype=torch.int32).cumsum(0, dtype=torch.int32)
    out = pe.flash_attention_varlen(q.cuda(), k.cuda(), v.cuda(), cu.cuda(), max(lengths), window, 0.125)
    torch.cuda.synchronize()
    assert out.shape == (1, total, heads * 64)
    ref, _ = oracle.attention(q[0].transpose(0, 1), k[0].transpose(0, 1), v[0].transpose(0, 1), cu, scale=0.125,
                              window=window)
    _assert_parity(out.view(total, heads, 64), ref, f"flash_attention_varlen w{window}")


@pytest.mark.parametrize("window", [(-1, -1), (64, 64)])
def test_rectangular_drop_ins(window):
    """ops.flash_attention (packed_encoders/ops.py:404-430): [B, H, S, D] views of an unpadded batch
    in, every row one sequence, [B, S, H*D] out; and attention_bshd's rectangular form ([B, S, H, D]
    in). Both against the oracle run per row."""
    pe = _b200()
    b, heads, s = 3, 4, 200
    gen = torch.Generator().manual_seed(31)
    qkv = torch.randn(b, s, 3, heads, 64, generator=gen).to(torch.bfloat16)
    q, k, v = (qkv[:, :, i].transpose(1, 2) for i in range(3))  # [B, H, S, D] views
    out = pe.flash_attention(q.cuda(), k.cuda(), v.cuda(), window, 0.125)
    dq, dk, dv = (qkv[:, :, i].cuda() for i in range(3))  # [B, S, H, D] strided views
    out_bshd = pe.attention_bshd(dq, dk, dv, window=window, scaling=0.125)
    torch.cuda.synchronize()
    assert out.shape == (b, s, heads * 64) and out_bshd.shape == (b, s, heads * 64)
    cu = torch.arange(0, (b + 1) * s, s, dtype=torch.int32)
    flat = [qkv[:, :, i].reshape(b * s, heads, 64) for i in range(3)]
    ref, _ = oracle.attention(*flat, cu, scale=0.125, window=window)
    _assert_parity(out.reshape(b * s, heads, 64), ref, f"flash_attention w{window}")
    _assert_parity(out_bshd.reshape(b * s, heads, 64), ref, f"attention_bshd rectangular w{window}")


@pytest.mark.parametrize("logit_scale", [0.01, 1.0, 8.0])
def test_softmax_stability_and_determinism(logit_scale):
    """tests/test_packed_short_attention.py:97-109: finite at extreme logit scales and bitwise
    repeatable."""
    pe = _b200()
    q, k, v, cu = packed_inputs([33, 65, 127], 12, 64, seed=11, logit_scale=logit_scale, device="cuda")
    a = pe.packed_short_attention(q, k, v, cu, 127, half_window=64, softmax_scale=0.125)
    b = pe.packed_short_attention(q, k, v, cu, 127, half_window=64, softmax_scale=0.125)
    assert torch.isfinite(a).all()
    assert torch.equal(a, b)
    ref, _ = oracle.attention(q, k, v, cu, scale=0.125, window=(64, 64))
    _assert_parity(a, ref, f"logit scale {logit_scale}")


def test_no_cross_sequence_leakage():
    """tests/test_packed_short_attention.py:112-126: neighbours' K/V scaled by 100 change nothing."""
    pe = _b200()
    for lengths in ([31, 65], [31, 65, 700], [700, 31]):
        q, k, v, cu = packed_inputs(lengths, 12, 64, seed=7, device="cuda")
        base = pe.packed_attention(q, k, v, cu, max(lengths), scale=0.125)
        k2, v2 = k.clone(), v.clone()
        k2[lengths[0]:] *= 100
        v2[lengths[0]:] *= -100
        changed = pe.packed_attention(q, k2, v2, cu, max(lengths), scale=0.125)
        assert torch.equal(base[:lengths[0]], changed[:lengths[0]])


def test_strided_v_view_like_modernbert():
    """v as a strided slice of a fused qkv projection (forward.py:201, ops.py:497)."""
    pe = _b200()
    lengths = [40, 200, 7]
    total, heads, dim = sum(lengths), 12, 64
    gen = torch.Generator().manual_seed(3)
    qkv = torch.randn(total, 3 * heads * dim, generator=gen).to(torch.bfloat16)
    cu = torch.tensor([0, 40, 240, 247], dtype=torch.int32)
    view = qkv.view(total, 3, heads, dim)
    q, k, v = view[:, 0], view[:, 1], view[:, 2]
    out = pe.packed_attention(q.cuda().contiguous(), k.cuda().contiguous(), qkv.cuda().view(total, 3, heads, dim)[:, 2],
                              cu.cuda(), 200, scale=0.125, window=(64, 64))
    ref, _ = oracle.attention(q, k, v, cu, scale=0.125, window=(64, 64))
    _assert_parity(out, ref, "strided v")


@pytest.mark.parametrize("window,causal", [((-1, -1), False), ((64, 64), False), ((-1, -1), True)])
def test_schedule_covers_every_block_once_with_sequences_contiguous(window, causal):
    """The device tile schedule: every 128-row query block of every sequence appears exactly once;
    the blocks of one long sequence are contiguous and in order (so concurrently running CTAs share
    its K/V in L2); groups are ordered longest-first (LPT)."""
    import packed_encoders_b200 as pe

    lengths = [3000, 7, 129, 0, 40, 1000, 90, 2000, 1, 300, 64, 65, 500]
    q, k, _, cu = packed_inputs(lengths, 2, 64, seed=5, device="cuda")
    plan = pe.ops.plan_attention(q, k, cu, max(lengths), window=window, causal=causal)
    torch.cuda.synchronize()
    ws = plan.workspace.cpu().view(torch.int32)
    n_items = int(ws[0])
    items = ws[64:64 + 4 * n_items].view(-1, 4).tolist()  # header is 256 bytes
    seen = {}
    for pos, (first, count, qb, cost) in enumerate(items):
        for s in range(first, first + count):
            if count > 1:
                assert lengths[s] <= 128
            seen.setdefault(s, []).append((pos, qb))
    for s, n in enumerate(lengths):
        if n == 0:
            continue
        blocks = seen[s]
        if n > 128:
            assert [qb for _, qb in blocks] == list(range((n + 127) // 128))
            positions = [pos for pos, _ in blocks]
            assert positions == list(range(positions[0], positions[0] + len(positions)))
        else:
            assert len(blocks) == 1
    group_cost = []
    for first, count, qb, cost in items:
        if qb == 0:
            group_cost.append(cost)
        else:
            group_cost[-1] = max(group_cost[-1], cost)
    assert group_cost == sorted(group_cost, reverse=True)


@pytest.mark.parametrize("mode", ["pass", "fused"])
@pytest.mark.parametrize("dim,window,causal,heads,kv_heads", [
    (64, (-1, -1), False, 4, 4), (64, (64, 64), False, 4, 4), (128, (-1, -1), True, 4, 2), (256, (-1, -1), True, 8, 2)])
def test_output_gate_matches_unfused(dim, window, causal, heads, kv_heads, mode, monkeypatch):
    """Output gate (the library's gate pass, and the fused epilogue) == attention then the
    reference's gate roundings: bf16(o * bf16(sigmoid(g))) (packed_encoders/_kernels/hybrid.py:196-205).
    The gate is a strided view, as when it comes out of a fused projection."""
    import packed_encoders_b200 as pe

    monkeypatch.setenv("PE_B200_GATE", mode)

    lengths = [300, 7, 129, 1000, 64, 1]
    q, k, v, cu = packed_inputs(lengths, heads, dim, kv_heads=kv_heads, seed=3, device="cuda")
    g_full = torch.randn(q.shape[0], heads, 2 * dim, device="cuda", generator=torch.Generator("cuda").manual_seed(4))
    gate = (g_full * 3).to(torch.bfloat16)[:, :, dim:]
    kw = dict(scale=dim ** -0.5, window=window, causal=causal)
    plain = pe.packed_attention(q, k, v, cu, max(lengths), **kw)
    fused = pe.packed_attention(q, k, v, cu, max(lengths), gate=gate, **kw)
    ref = (plain.float() * torch.sigmoid(gate.float()).to(torch.bfloat16).float()).to(torch.bfloat16)
    diff = (fused.float() - ref.float()).abs()
    assert torch.isfinite(fused.float()).all()
    # identical roundings; a sigmoid value within an ulp of a bf16 rounding boundary may round the other way
    assert diff.max().item() <= 2e-2
    assert (diff > 0).float().mean().item() < 0.01
    assert pe.device_error_word() == 0


def test_cuda_graph_capture_replays_new_lengths():
    """Graph capture (the reference captures its packed forward, graph.py:8-18; no host syncs and
    no host reads of cu_seqlens): a global and a windowed call captured once replay correctly after
    new sequence lengths (same count and total) are written into the captured cu_seqlens buffer,
    because the tile schedule is rebuilt on the device inside the graph."""
    pe = _b200()
    lengths_a, lengths_b = [300, 7, 129, 1000, 64], [100, 400, 1, 900, 99]
    assert sum(lengths_a) == sum(lengths_b)
    q, k, v, cu_a = packed_inputs(lengths_a, 4, 64, seed=21, device="cuda")
    cu_b = torch.tensor([0] + lengths_b, dtype=torch.int32, device="cuda").cumsum(0, dtype=torch.int32)
    cu = cu_a.clone()
    bound = 1024  # a host-side upper bound on the lengths, as a graph runner passes
    outs = [torch.empty_like(q), torch.empty_like(q)]
    windows = [(-1, -1), (64, 64)]

    def step():
        for out, window in zip(outs, windows):
            pe.packed_attention(q, k, v, cu, bound, scale=0.125, window=window, out=out)

    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        step()  # warm-up on the capture stream (its workspace is allocated here, not during capture)
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=side):
        step()
    for new_cu in (cu_a, cu_b, cu_a):
        cu.copy_(new_cu)
        graph.replay()
        torch.cuda.synchronize()
        for out, window in zip(outs, windows):
            eager = pe.packed_attention(q, k, v, new_cu, bound, scale=0.125, window=window)
            assert torch.equal(out, eager), window
    assert pe.device_error_word() == 0


@pytest.mark.parametrize("name", rope_golden_names())
def test_rope_golden_vectors(name):
    """Fused RoPE against the reference's own pipeline: its CPU RoPE (cpu/attention.py:281-303)
    on un-rotated q/k, then its native attention (fixtures from tests/golden/make_golden.py)."""
    pe = _b200()
    g = load_rope_golden(name)
    lengths = (g["cu_q"][1:] - g["cu_q"][:-1]).tolist()
    out = pe.packed_attention(g["q"].cuda(), g["k"].cuda(), g["v"].cuda(), g["cu_q"].cuda(), max(lengths),
                              scale=g["scale"], window=g["window"], rope=(g["cos"].cuda(), g["sin"].cuda()))
    torch.cuda.synchronize()
    _assert_parity(out, g["out"], name)
    assert pe.device_error_word() == 0


ROPE_CASES = [
    # (lengths, heads, kv_heads, window, causal)
    ([300, 7, 129, 1000, 64, 1], 4, 4, (-1, -1), False),
    ([300, 7, 129, 1000, 64, 1], 4, 4, (64, 64), False),
    ([30] * 40 + [5, 100], 12, 12, (-1, -1), False),
    ([700, 3, 260], 4, 2, (-1, -1), True),
    ([17, 250, 9, 0, 128], 4, 1, (16, 3), False),
]


@pytest.mark.parametrize("lengths,heads,kv_heads,window,causal", ROPE_CASES)
def test_fused_rope_matches_rotate_then_attend(lengths, heads, kv_heads, window, causal):
    """Fused RoPE == the oracle's rotation of q and k followed by attention (parity bars), and ==
    this library's unfused path on the same rotated inputs up to rare last-bit differences of the
    rotation's rounding."""
    pe = _b200()
    q, k, v, cu = packed_inputs(lengths, heads, 64, kv_heads=kv_heads, seed=31)
    cos, sin = rope_tables(lengths, theta=160000.0 if window == (-1, -1) else 10000.0)
    rq, rk = oracle.rope_bshd(q, cos, sin), oracle.rope_bshd(k, cos, sin)
    ref, _ = oracle.attention(rq, rk, v, cu, scale=0.125, window=window, causal=causal)
    kw = dict(scale=0.125, window=window, causal=causal)
    out = pe.packed_attention(q.cuda(), k.cuda(), v.cuda(), cu.cuda(), max(lengths), rope=(cos.cuda(), sin.cuda()), **kw)
    unfused = pe.packed_attention(rq.cuda(), rk.cuda(), v.cuda(), cu.cuda(), max(lengths), **kw)
    torch.cuda.synchronize()
    _assert_parity(out, ref, f"rope {lengths[:6]} H{heads}/{kv_heads} w{window} c{causal}")
    assert (out != unfused).float().mean().item() < 0.01
    assert pe.device_error_word() == 0


def test_fused_rope_on_qkv_views():
    """q and k as strided views of a fused qkv projection [T, 3, H, D] (forward.py:197-205), windowed
    and global, with strided table views."""
    pe = _b200()
    lengths, heads = [40, 200, 7, 513], 12
    total = sum(lengths)
    gen = torch.Generator().manual_seed(9)
    qkv = torch.randn(total, 3, heads, 64, generator=gen).to(torch.bfloat16)
    cos, sin = rope_tables(lengths)
    tables = torch.stack((cos, sin), 1)  # [T, 2, D]: each table a view with row stride 2*D
    cu = torch.tensor([0] + lengths, dtype=torch.int32).cumsum(0, dtype=torch.int32)
    for window in ((64, 64), (-1, -1)):
        out = pe.packed_attention(qkv.cuda()[:, 0], qkv.cuda()[:, 1], qkv.cuda()[:, 2], cu.cuda(), max(lengths),
                                  scale=0.125, window=window, rope=(tables.cuda()[:, 0], tables.cuda()[:, 1]))
        rq, rk = oracle.rope_bshd(qkv[:, 0], cos, sin), oracle.rope_bshd(qkv[:, 1], cos, sin)
        ref, _ = oracle.attention(rq, rk, qkv[:, 2].contiguous(), cu, scale=0.125, window=window)
        _assert_parity(out, ref, f"rope qkv views {window}")
    assert pe.device_error_word() == 0



@pytest.mark.parametrize("dense", [False, True])
def test_apply_rope_bshd_matches_oracle(dense):
    """The standalone RoPE pass (the reference's apply_rope_bshd signature, _kernels/rope.py:302-345)
    against the oracle's rotate-half restatement: per-token gathered tables of a packed batch, and
    one dense [S, D] table over a [B, S] batch (row t % S)."""
    pe = _b200()
    heads, d = 12, 64
    gen = torch.Generator().manual_seed(13)
    if dense:
        b, s = 3, 200
        qkv = torch.randn(b, s, 3 * heads * d, generator=gen).to(torch.bfloat16)
        cos, sin = rope_tables([s], theta=160000.0)
        rows_cos, rows_sin = cos.repeat(b, 1), sin.repeat(b, 1)
    else:
        lengths = [7, 300, 1, 129]
        qkv = torch.randn(1, sum(lengths), 3 * heads * d, generator=gen).to(torch.bfloat16)
        cos, sin = rope_tables(lengths)
        rows_cos, rows_sin = cos, sin
    q, k = pe.apply_rope_bshd(qkv.cuda(), heads, d, cos.cuda(), sin.cuda())
    assert q.shape == qkv.shape[:-1] + (heads, d) and q.is_contiguous() and k.is_contiguous()
    flat = qkv.reshape(-1, 3, heads, d)
    for got, x in ((q, flat[:, 0]), (k, flat[:, 1])):
        ref = oracle.rope_bshd(x, rows_cos, rows_sin)
        got = got.reshape(-1, heads, d).cpu()
        diff = (got.float() - ref.float()).abs()
        assert (diff <= ref.float().abs() * 2.0 ** -7 + 1e-6).all()  # at most one bf16 rounding apart
        assert (got != ref).float().mean().item() < 0.01
