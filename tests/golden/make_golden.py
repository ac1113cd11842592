"""Generate the golden fixtures in tests/golden/ from the reference implementation itself.

Run in a container where the reference tree (packed-encoders 0.3.0) is importable:

    PACKED_ENCODERS_CPU_CACHE_DIR= PYTHONPATH=<reference checkout> python tests/golden/make_golden.py

Every expected output below is produced by the REFERENCE's own code path, never by this
repository's oracle:

- ``native_*``: ``packed_encoders.cpu.attention.CPUAttention._native`` (its x86 C kernel
  ``pe_local_attention``, compiled by the reference's own loader), fp32, head_dim 64,
  scale 0.125; lengths and edge rows from tests/test_packed_short_attention.py:68-71,
  tests/test_cpu_short_attention.py:197-201, tests/test_modernbert_cpu.py:302-321,527-551.
- ``segments_*``: ``packed_encoders.runtime.attention._reference`` (fp32 per-segment SDPA,
  runtime/attention.py:202-204) on the probe geometry of runtime/attention.py:216 and the
  Qwen3.5 attention geometry 8/2/256 (tests/test_qwen35.py:136-152).
- ``prefixed_*``: ``runtime.attention.reference_prefixed`` (runtime/attention.py:242-244)
  on the prefixed probe lengths of runtime/attention.py:250.
- ``rope_*``: ``CPUAttention.rope_layout`` (cpu/attention.py:281-303) then ``_native``: RoPE'd
  attention from un-rotated q/k and per-token tables (see ``rope_cases``).

The reference returns no log-sum-exp, so the fixtures carry none; LSE is checked against
the oracle's definition (natural log of the softmax denominator) in the tests.

Inputs are stored as bf16 bit patterns (what the GPU consumes); the reference ran on the
same values upcast to fp32.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def _bf16(shape, gen, scale=1.0):
    return (torch.randn(*shape, generator=gen) * scale).to(torch.bfloat16)


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def _cu(lengths):
    return np.concatenate([[0], np.cumsum(lengths)]).astype(np.int32)


def _save(name, *, q, k, v, lengths, out, scale, window, causal, lengths_k=None, note=""):
    path = HERE / f"{name}.npz"
    np.savez_compressed(
        path, q=_bits(q), k=_bits(k), v=_bits(v), cu_q=_cu(lengths),
        cu_k=_cu(lengths if lengths_k is None else lengths_k),
        out=out.detach().to(torch.float32).contiguous().numpy(),
        scale=np.float32(scale), window=np.array(window, dtype=np.int32), causal=np.int32(bool(causal)),
        note=np.array(note),
    )
    print(f"{path.name}: T={q.shape[0]} H={q.shape[1]} KV={k.shape[1]} D={q.shape[2]} "
          f"window={window} causal={causal} bytes={path.stat().st_size}")


def native_cases():
    from packed_encoders.cpu.attention import CPUAttention

    engine = CPUAttention("native", 64, 64, 4)
    if engine.library is None:
        raise SystemExit("reference native CPU attention did not build")

    def run(name, lengths, heads, half, seed, edge_rows=False, scale=1.0, note=""):
        gen = torch.Generator().manual_seed(seed)
        total = sum(lengths)
        q, k, v = (_bf16((total, heads, 64), gen, scale) for _ in range(3))
        if edge_rows:
            q[0].zero_()          # uniform logits (ties)
            q[1] = (q[1].float() * 100).to(torch.bfloat16)   # one very sharp row (exp underflow)
        # The reference kernel is head-major [1, H, T, 64].
        qh, kh, vh = (t.float().permute(1, 0, 2).unsqueeze(0).contiguous() for t in (q, k, v))
        boundaries = torch.tensor(lengths, dtype=torch.int32)
        out = engine._native(qh, kh, vh, tuple(lengths), boundaries, half).clone()  # [1,H,T,64]
        out = out.squeeze(0).permute(1, 0, 2).contiguous()
        window = (-1, -1) if half >= max(lengths) else (half, half)
        _save(name, q=q, k=k, v=v, lengths=lengths, out=out, scale=0.125, window=window, causal=False,
              note=note)

    ragged = [1, 2, 31, 32, 33, 63, 64, 65, 127, 128]
    run("native_ragged_global", ragged, 1, max(ragged), 17, note="test_packed_short_attention.py:68")
    run("native_ragged_local64", ragged, 1, 64, 17, note="test_packed_short_attention.py:68")
    edge = [16, 32, 1, 15, 17, 31, 33, 65]
    for half in (0, 15, 64):
        run(f"native_edge_half{half}", edge, 3, half, 43, edge_rows=True, scale=2.0,
            note="test_cpu_short_attention.py:197-201")
    run("native_modernbert_local", [7, 65, 66, 1, 130, 200], 2, 64, 3, note="test_modernbert_cpu.py:302-321")
    mixed = [17, 1, 8, 3, 65, 2, 128]
    run("native_modernbert_global", mixed, 2, max(mixed), 4, note="test_modernbert_cpu.py:527-551")
    run("native_long_local", [129, 1, 2, 300], 2, 64, 5, note="test_modernbert_cpu.py:545 (129,1,2)")


def segment_cases():
    from packed_encoders.runtime.attention import _reference, reference_prefixed

    def run(name, lengths, heads, kv_heads, dim, causal, window, scale, seed, note):
        gen = torch.Generator().manual_seed(seed)
        total = sum(lengths)
        q = _bf16((total, heads, dim), gen)
        k = _bf16((total, kv_heads, dim), gen)
        v = _bf16((total, kv_heads, dim), gen)
        out = _reference(q, k, v, lengths, causal, window, scale)
        _save(name, q=q, k=k, v=v, lengths=lengths, out=out,
              scale=dim ** -0.5 if scale is None else scale, window=window, causal=causal, note=note)

    probe = [5, 64, 0, 37]
    run("segments_gqa256_causal", probe, 8, 2, 256, True, (-1, -1), None, 0,
        "runtime/attention.py:216 probe lengths; Qwen3.5 geometry tests/test_qwen35.py:136-152")
    run("segments_gqa256_bidir", probe, 4, 1, 256, False, (-1, -1), None, 1,
        "runtime/attention.py:216 probe lengths, bidirectional")
    run("segments_window16_gqa64", [5, 35, 0, 37, 130], 4, 1, 64, False, (16, 16), 0.125, 2,
        "runtime/attention.py:209-216 windowed probe (span 2*16+3)")
    run("segments_causal_window_left8", [5, 40, 0, 19], 4, 2, 64, True, (8, -1), None, 3,
        "runtime/attention.py:157-170 causal band with a left window")

    gen = torch.Generator().manual_seed(1)
    lq, lk = [5, 1, 37, 16], [40, 64, 37, 80]
    q = _bf16((sum(lq), 8, 256), gen)
    k = _bf16((sum(lk), 2, 256), gen)
    v = _bf16((sum(lk), 2, 256), gen)
    out = reference_prefixed(q, k, v, lq, lk, True, (-1, -1), None)
    _save("prefixed_gqa256_causal", q=q, k=k, v=v, lengths=lq, lengths_k=lk, out=out, scale=256 ** -0.5,
          window=(-1, -1), causal=True, note="runtime/attention.py:250 prefixed probe lengths")


def rope_tables(lengths, theta, dim=64):
    """Per-token gathered RoPE tables [T, dim] (positions restart at 0 in every sequence;
    ModernBERT's rotary embedding: inverse frequencies theta^(-2i/dim), emb = [freqs, freqs])."""
    inv = 1.0 / theta ** (torch.arange(0, dim, 2, dtype=torch.float32) / dim)
    pos = torch.cat([torch.arange(n, dtype=torch.float32) for n in lengths])
    freqs = pos[:, None] * inv[None, :]
    emb = torch.cat((freqs, freqs), -1)
    return emb.cos().to(torch.bfloat16), emb.sin().to(torch.bfloat16)


def rope_cases():
    """``rope_*``: the reference's CPU RoPE (``CPUAttention.rope_layout``, cpu/attention.py:281-303,
    rotate-half in fp32) on un-rotated q/k from a packed qkv, then its native attention on the
    rotated q/k. The fixtures keep q/k un-rotated plus the bf16 tables, the reference's rotated q/k
    (fp32) and its attention output."""
    from packed_encoders.cpu.attention import CPUAttention

    engine = CPUAttention("native", 64, 64, 4)
    if engine.library is None:
        raise SystemExit("reference native CPU attention did not build")

    def run(name, lengths, heads, half, theta, seed, note):
        gen = torch.Generator().manual_seed(seed)
        total = sum(lengths)
        q, k, v = (_bf16((total, heads, 64), gen) for _ in range(3))
        cos, sin = rope_tables(lengths, theta)
        qkv = torch.stack((q, k, v), 1).float().reshape(1, total, 3 * heads * 64).contiguous()
        rq, rk, rv = (t.clone().contiguous() for t in
                      engine.rope_layout(qkv, cos.float()[None, None].contiguous(), sin.float()[None, None].contiguous(),
                                         heads, 64))
        boundaries = torch.tensor(lengths, dtype=torch.int32)
        out = engine._native(rq, rk, rv, tuple(lengths), boundaries, half).clone()
        out = out.squeeze(0).permute(1, 0, 2).contiguous()
        window = (-1, -1) if half >= max(lengths) else (half, half)
        path = HERE / f"{name}.npz"
        np.savez_compressed(
            path, q=_bits(q), k=_bits(k), v=_bits(v), cos=_bits(cos), sin=_bits(sin), cu_q=_cu(lengths),
            cu_k=_cu(lengths), out=out.to(torch.float32).numpy(),
            rq=rq.squeeze(0).permute(1, 0, 2).contiguous().numpy(), rk=rk.squeeze(0).permute(1, 0, 2).contiguous().numpy(),
            scale=np.float32(0.125), window=np.array(window, dtype=np.int32), causal=np.int32(0), note=np.array(note),
        )
        print(f"{path.name}: T={total} H={heads} window={window} theta={theta} bytes={path.stat().st_size}")

    run("rope_native_local", [7, 65, 66, 1, 130, 200], 1, 64, 10000.0, 6,
        "test_modernbert_cpu.py:302-321 lengths; local layers, RoPE theta 10000")
    run("rope_native_global", [17, 1, 8, 3, 65, 2, 128, 300], 1, 300, 160000.0, 7,
        "test_modernbert_cpu.py:527-551 lengths + 300; global layers, RoPE theta 160000")


if __name__ == "__main__":
    try:
        import packed_encoders  # noqa: F401
    except ImportError:
        sys.exit("packed_encoders (the reference) must be importable: put its checkout on PYTHONPATH")
    torch.set_num_threads(4)
    only = sys.argv[1:]
    with torch.inference_mode():
        if not only or "native" in only:
            native_cases()
        if not only or "segments" in only:
            segment_cases()
        if not only or "rope" in only:
            rope_cases()
