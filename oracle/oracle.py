"""TEST INFRASTRUCTURE ONLY: ctypes bindings for the CPU oracle.

Two libraries:

- ``oracle/liboracle.so`` (``attention_oracle.c``): this repository's fp32 restatement
  of the reference's packed attention (windows, causal, GQA, prefixed segments, LSE).
- ``oracle/_ref/libref_attn_v{4,3}.so``: the reference's OWN CPU kernel,
  ``pe_local_attention`` from packed_encoders/cpu/local_attention_x86.c:192-235 of
  packed-encoders 0.3.0, compiled from the reference tree by ``oracle/Makefile``. It is
  head-major ``[H, T, 64]``, fixed scale 0.125 (:55), half-window ``half`` (global when
  ``half >= max length``, :206), lengths >= 1 (:201).

The product never imports this module. Callers: tests, ``__graft_entry__.smoke`` and
``bench.py`` (CPU baseline / reference arm).
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from functools import lru_cache
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
_LIB = HERE / "liboracle.so"
_REF = {"v4": HERE / "_ref" / "libref_attn_v4.so", "v3": HERE / "_ref" / "libref_attn_v3.so"}

_c_long = ctypes.c_long
_c_int = ctypes.c_int
_ptr = ctypes.c_void_p


def build(reference: bool | None = None) -> None:
    """Compile the oracle (and the reference kernel when the reference tree exists)."""
    from oracle.reference_tree import reference_dir

    targets = ["all"]
    tree = reference_dir()
    if reference is None:
        reference = tree is not None and (tree / "packed_encoders/cpu/local_attention_x86.c").exists()
    if reference:
        targets += ["ref", f"REFERENCE={tree}"]
    subprocess.run(["make", "-s", "-C", str(HERE), *targets], check=True)


@lru_cache(maxsize=1)
def _lib():
    if not _LIB.exists():
        build(reference=False)
    lib = ctypes.CDLL(str(_LIB))
    fn = lib.oracle_attention_prefixed
    fn.argtypes = ([_ptr] * 7 + [_c_int] * 6 + [_c_long] * 8
                   + [ctypes.c_float, _c_int, _c_int, _c_int, _c_int])
    fn.restype = _c_int
    fn = lib.oracle_useful_pairs
    fn.argtypes = [_ptr, _c_int, _c_int, _c_int, _c_int]
    fn.restype = ctypes.c_longlong
    return lib


def _cpu_flags() -> set[str]:
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("flags"):
                    return set(line.split(":", 1)[1].split())
    except OSError:
        pass
    return set()


def available_reference() -> str | None:
    """Which build of the reference kernel this host can run ('v4', 'v3') or None."""
    flags = _cpu_flags()
    if _REF["v4"].exists() and {"avx512f", "avx512bw", "avx512dq", "avx512vl"} <= flags:
        return "v4"
    if _REF["v3"].exists() and {"avx2", "fma"} <= flags:
        return "v3"
    return None


@lru_cache(maxsize=1)
def _ref_lib():
    level = available_reference()
    if level is None:
        raise RuntimeError("reference CPU attention not built for this host (make -C oracle ref)")
    lib = ctypes.CDLL(str(_REF[level]))
    fn = lib.pe_local_attention
    # local_attention_x86.c:192-194 and the reference's own ctypes signature,
    # packed_encoders/cpu/attention.py:47-49.
    fn.argtypes = [_ptr] * 5 + [_c_int] * 7 + [_ptr] * 2 + [ctypes.c_size_t]
    fn.restype = _c_int
    return lib


def default_threads() -> int:
    return max(1, len(os.sched_getaffinity(0)))


def _f32(t: torch.Tensor) -> torch.Tensor:
    t = t.detach().to("cpu", torch.float32)
    return t if t.stride(-1) == 1 else t.contiguous()


def attention_prefixed(q, k, v, cu_q, cu_k, *, scale, window=(-1, -1), causal=False, threads=None,
                       return_lse=True):
    """fp32 oracle: q [Tq,H,D], k/v [Tk,KV,D]; query segment s is the last
    ``len_q`` rows of key segment s. Returns (out [Tq,H,D] fp32, lse [H,Tq] fp32 or None)."""
    q, k, v = _f32(q), _f32(k), _f32(v)
    cu_q = cu_q.detach().to("cpu", torch.int32).contiguous()
    cu_k = cu_k.detach().to("cpu", torch.int32).contiguous()
    tq, heads, dim = q.shape
    tk, kv_heads, _ = k.shape
    out = torch.empty(tq, heads, dim, dtype=torch.float32)
    lse = torch.empty(heads, tq, dtype=torch.float32) if return_lse else None
    status = _lib().oracle_attention_prefixed(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), lse.data_ptr() if lse is not None else None,
        cu_q.data_ptr(), cu_k.data_ptr(), cu_q.numel() - 1, tq, tk, heads, kv_heads, dim,
        q.stride(0), q.stride(1), k.stride(0), k.stride(1), v.stride(0), v.stride(1),
        out.stride(0), out.stride(1), float(scale), int(window[0]), int(window[1]), int(bool(causal)),
        int(threads or default_threads()),
    )
    if status:
        raise ValueError(f"oracle_attention rejected its arguments (status {status})")
    return out, lse


def attention(q, k, v, cu_seqlens, *, scale, window=(-1, -1), causal=False, threads=None, return_lse=True):
    """fp32 oracle for the packed self-attention form (same boundaries for q and k)."""
    return attention_prefixed(q, k, v, cu_seqlens, cu_seqlens, scale=scale, window=window, causal=causal,
                              threads=threads, return_lse=return_lse)


def useful_pairs(cu_seqlens, *, window=(-1, -1), causal=False) -> int:
    """Allowed query-key pairs of one head, summed over segments."""
    cu = cu_seqlens.detach().to("cpu", torch.int32).contiguous()
    return int(_lib().oracle_useful_pairs(cu.data_ptr(), cu.numel() - 1, int(window[0]), int(window[1]),
                                          int(bool(causal))))


class _RefScratch:
    buffer: torch.Tensor | None = None


def reference_local_attention(q, k, v, lengths, half, *, token_major=False, threads=None, tile=64,
                              out=None):
    """Run the reference's own ``pe_local_attention`` (fp32, head-major [H,T,64] inputs).

    Mirrors ``CPUAttention._native_args`` (packed_encoders/cpu/attention.py:418-440):
    scratch of ``workers * (tile + 64) * columns`` floats, ``columns`` the window width
    rounded up to 16 keys.
    """
    q, k, v = (t.detach().to("cpu", torch.float32).contiguous() for t in (q, k, v))
    heads, tokens, dim = q.shape
    if dim != 64:
        raise ValueError("the reference CPU kernel is head_dim 64 only")
    lengths = [int(n) for n in lengths]
    workers = min(int(threads or default_threads()), heads * len(lengths))
    columns = -(-min(tile + 2 * half, max(lengths)) // 16) * 16
    needed = workers * (tile + 64) * columns
    if _RefScratch.buffer is None or _RefScratch.buffer.numel() < needed:
        _RefScratch.buffer = torch.empty(needed, dtype=torch.float32)
    scratch = _RefScratch.buffer
    boundaries = torch.tensor(lengths, dtype=torch.int32)
    shape = (tokens, heads * dim) if token_major else (heads, tokens, dim)
    if out is None or tuple(out.shape) != shape:
        out = torch.empty(shape, dtype=torch.float32)
    status = _ref_lib().pe_local_attention(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), boundaries.data_ptr(), tokens, heads,
        len(lengths), tile, int(half), int(bool(token_major)), workers, None, scratch.data_ptr(), scratch.numel(),
    )
    if status:
        raise ValueError(f"pe_local_attention failed: {status}")
    return out


def rope_bshd(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """Rotary embedding of ``x`` ``[T, H, D]`` with per-token tables ``[T, D]``, rotate-half
    pairing (dims d and d + D/2), in fp32, rounded to ``x``'s dtype. Restates the reference's
    ``t * cos + cat(-b, a) * sin`` (packed_encoders/cpu/attention.py:298-301) and its GPU
    kernel's rounding of the result to the input dtype (packed_encoders/_kernels/rope.py:5-6,
    190-197)."""
    xf = x.float()
    c = cos.float()[:, None, :]
    s = sin.float()[:, None, :]
    a, b = xf.chunk(2, -1)
    return (xf * c + torch.cat((-b, a), -1) * s).to(x.dtype)

