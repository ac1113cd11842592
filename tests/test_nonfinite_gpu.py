"""Non-finite inputs stay inside their own sequence (GPU).

A key tile's P.V multiplies every key row the tile holds: rows of neighbouring sequences in a
packed tile and rows past a segment's end, with P = 0. 0 x Inf is NaN, so the kernel recomputes a
non-finite output chunk from the row's own keys (attn_fwd.cu, recompute_chunk). The reference
computes each sequence on its own with masked loads (packed_encoders/_kernels/
triton_packed_attention.py:96-112, `other=0.0`), so a non-finite value there reaches only its own
sequence's queries. These tests poison V and K rows of one sequence and check that every other
sequence's output equals the clean call's within the parity bar and is finite, that the poisoned
sequence's attending rows carry the non-finite value in the poisoned column only, and that LSE
stays finite.
"""

from __future__ import annotations

import pytest
import torch

from conftest import packed_inputs

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-2


def _seq_of(cu, n_tokens):
    seq = torch.zeros(n_tokens, dtype=torch.long)
    for i, (a, b) in enumerate(zip(cu.tolist(), cu.tolist()[1:])):
        seq[a:b] = i
    return seq


CASES = [
    # name, lengths, heads, kv_heads, dim, window, causal, poisoned sequence
    ("packed-short-global", [17, 33, 8, 50, 21, 64, 9, 40, 12, 30], 4, 4, 64, (-1, -1), False, 3),
    ("packed-short-window", [17, 33, 8, 50, 21, 64, 9, 40, 12, 30], 4, 4, 64, (8, 8), False, 5),
    ("long-tail-global", [300, 200, 150], 4, 4, 64, (-1, -1), False, 1),
    ("long-tail-window", [300, 200, 150], 4, 4, 64, (64, 64), False, 1),
    ("d128", [130, 70, 90], 4, 4, 128, (-1, -1), False, 1),
    ("d256-gqa-causal", [130, 70, 90], 8, 2, 256, (-1, -1), True, 1),
]


@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
@pytest.mark.parametrize("poison", ["v_inf", "v_nan", "k_inf"])
def test_nonfinite_rows_stay_in_their_sequence(case, poison):
    import packed_encoders_b200 as pe

    name, lengths, heads, kv_heads, dim, window, causal, bad_seq = case
    q, k, v, cu = packed_inputs(lengths, heads, dim, kv_heads=kv_heads, seed=71, device="cuda")
    scale = dim ** -0.5
    kw = dict(scale=scale, window=window, causal=causal, return_lse=True)
    clean, clean_lse = pe.packed_attention(q, k, v, cu, max(lengths), **kw)

    # The poisoned token is the FIRST of its sequence: for long sequences it sits in the last key
    # tile of the sequence before it, for packed ones in the same tile as its neighbours.
    tok = int(cu[bad_seq])
    kvh, col = kv_heads - 1, dim // 2 + 3
    if poison == "k_inf":
        k = k.clone()
        k[tok, kvh, col] = float("inf")
    else:
        v = v.clone()
        v[tok, kvh, col] = float("inf") if poison == "v_inf" else float("nan")
    out, lse = pe.packed_attention(q, k, v, cu, max(lengths), **kw)
    torch.cuda.synchronize()

    seq = _seq_of(cu.cpu(), q.shape[0]).to("cuda")
    other = seq != bad_seq
    o, c = out[other].float(), clean[other].float()
    assert torch.isfinite(o).all(), f"{name}/{poison}: non-finite output leaked into other sequences"
    err = (o - c).abs().max().item()
    print(f"PARITY nonfinite {name} {poison}: other-sequence max_abs vs clean {err:.5f}")
    assert err <= MAX_ABS
    assert torch.isfinite(lse[:, other]).all()
    if poison != "k_inf":
        group = heads // kv_heads
        heads_of_kvh = list(range(kvh * group, (kvh + 1) * group))
        mine = (seq == bad_seq).nonzero().flatten()
        pos = mine - tok
        rel = pos  # query position minus the poisoned key's position (0)
        attends = torch.ones_like(pos, dtype=torch.bool)
        if window[0] >= 0:
            attends &= rel <= window[0]
        if window[1] >= 0:
            attends &= rel >= -window[1]
        rows = mine[attends]
        bad = out[rows][:, heads_of_kvh, col].float()
        assert not torch.isfinite(bad).any(), f"{name}/{poison}: the attending rows lost the non-finite value"
        # everything else of the poisoned sequence: finite and equal to the clean call
        keep = torch.ones(out.shape[1:], dtype=torch.bool, device="cuda")
        keep[heads_of_kvh, col] = False
        mo, mc = out[mine].float()[:, keep], clean[mine].float()[:, keep]
        assert torch.isfinite(mo).all()
        assert (mo - mc).abs().max().item() <= MAX_ABS
