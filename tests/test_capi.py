"""The C-ABI library loads on CPU and exports every symbol include/*.h declares; host-side
argument validation (no CUDA calls) behaves as documented."""

from __future__ import annotations

import ctypes
import re
import subprocess
from pathlib import Path

import pytest

from packed_encoders_b200 import _lib
from packed_encoders_b200.build import LIB, build

ROOT = Path(__file__).resolve().parents[1]


def _declared_symbols() -> set[str]:
    names = set()
    for header in (ROOT / "include").glob("*.h"):
        text = header.read_text()
        names |= set(re.findall(r"^\s*(?:int|const char\*|void)\s+(pe_b200_\w+)\s*\(", text, flags=re.M))
    return names


def test_library_exports_every_declared_symbol():
    build()
    out = subprocess.run(["nm", "-D", "--defined-only", str(LIB)], check=True, capture_output=True, text=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if line.strip()}
    declared = _declared_symbols()
    assert declared, "no declarations parsed from include/*.h"
    assert declared <= exported, f"missing exports: {sorted(declared - exported)}"
    assert set(_lib.EXPORTS) <= declared


def test_abi_version_and_status_strings():
    so = _lib.lib()
    assert so.pe_b200_abi_version() == _lib.ABI_VERSION
    assert _lib.status_string(0) == "ok"
    assert "head_dim" in _lib.status_string(-8)


def _params(**kw):
    base = dict(n_seq=4, total_q=1000, total_k=1000, max_seqlen_q=600, max_seqlen_k=600, heads=12, kv_heads=12,
                head_dim=64, scale=0.125, window_left=-1, window_right=-1, causal=0)
    base.update(kw)
    return _lib.PeB200AttnParams(**base)


def _size(p):
    n = ctypes.c_size_t(0)
    status = _lib.lib().pe_b200_attn_workspace_size(ctypes.byref(p), ctypes.byref(n))
    return status, n.value


def test_workspace_size_and_validation():
    status, n = _size(_params())
    assert status == 0 and n >= 256 + 16 * (4 + 1000 // 128)
    assert _size(_params(head_dim=96))[0] == -8     # PE_B200_ERR_UNSUPPORTED
    assert _size(_params(heads=12, kv_heads=5))[0] == -2  # PE_B200_ERR_SHAPE
    assert _size(_params(window_left=-2))[0] == -4   # PE_B200_ERR_WINDOW
    assert _size(_params(total_k=0))[0] == -2


@pytest.mark.parametrize("struct", ["PeB200AttnParams", "PeB200AttnBwdParams"])
def test_struct_layout_matches_header(tmp_path, struct):
    """The ctypes mirror has the C compiler's offsets for every field of the parameter blocks."""
    P = getattr(_lib, struct)
    names = [f[0] for f in P._fields_]
    src = tmp_path / "layout.c"
    src.write_text('#include <stdio.h>\n#include <stddef.h>\n#include "pe_b200_attn.h"\nint main(void) {\n'
                   + "".join(f'  printf("%zu\\n", offsetof({struct}, {n}));\n' for n in names)
                   + f'  printf("%zu\\n", sizeof({struct}));\n  return 0;\n}}\n')
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-I", str(ROOT / "include"), str(src), "-o", str(exe)], check=True)
    c_offsets = [int(x) for x in subprocess.run([str(exe)], check=True, capture_output=True,
                                                text=True).stdout.split()]
    assert c_offsets[:-1] == [getattr(P, n).offset for n in names]
    assert c_offsets[-1] == ctypes.sizeof(P)


def test_backward_validation_without_touching_cuda():
    """The backward's host checks: head_dim 64 only, workspace size and alignment, strides."""
    P = _lib.PeB200AttnBwdParams
    so = _lib.lib()

    def size(**kw):
        base = dict(n_seq=3, total=500, max_seqlen=300, heads=4, head_dim=64, scale=0.125, window_left=-1,
                    window_right=-1, causal=0)
        base.update(kw)
        n = ctypes.c_size_t(0)
        return so.pe_b200_attn_bwd_workspace_size(ctypes.byref(P(**base)), ctypes.byref(n)), n.value

    status, n = size()
    assert status == 0 and n >= 500 * 4 * 64 * 4 + 2 * 500 * 4 * 4
    assert size(head_dim=128)[0] == -8
    assert size(window_left=-3)[0] == -4
    full = dict(n_seq=3, total=500, max_seqlen=300, heads=4, head_dim=64, scale=0.125, window_left=-1,
                window_right=-1, causal=0, q=16, k=16, v=16, out=16, dout=16, lse=16, dq=16, dk=16, dv=16,
                cu_seqlens=16, workspace=256, workspace_bytes=n)
    for prefix in ("q", "k", "v", "o", "do", "dq", "dk", "dv"):
        full[f"{prefix}_stride_token"], full[f"{prefix}_stride_head"] = 256, 64
    assert so.pe_b200_attn_bwd(ctypes.byref(P(**{**full, "workspace_bytes": n - 1})), None) == -5
    assert so.pe_b200_attn_bwd(ctypes.byref(P(**{**full, "workspace": 128})), None) == -5
    assert so.pe_b200_attn_bwd(ctypes.byref(P(**{**full, "dk": 24})), None) == -3
    assert so.pe_b200_attn_bwd(ctypes.byref(P(**{**full, "dv_stride_token": 4})), None) == -3
    assert so.pe_b200_attn_bwd(ctypes.byref(P(**{**full, "lse": None})), None) == -1


def test_gate_stride_validation_without_touching_cuda():
    """A gate whose address or strides break the 16-byte rule is rejected before any CUDA call."""
    base = dict(q=16, k=16, v=16, out=16, cu_seqlens_q=16, cu_seqlens_k=16, workspace=256, workspace_bytes=1 << 20,
                q_stride_token=768, q_stride_head=64, k_stride_token=768, k_stride_head=64, v_stride_token=768,
                v_stride_head=64, o_stride_token=768, o_stride_head=64)
    so = _lib.lib()
    assert so.pe_b200_attn_fwd(ctypes.byref(_params(**base, gate=24, g_stride_token=768, g_stride_head=64)), None) == -3
    assert so.pe_b200_attn_fwd(ctypes.byref(_params(**base, gate=32, g_stride_token=770, g_stride_head=64)), None) == -3
    assert so.pe_b200_attn_fwd(ctypes.byref(_params(**base, gate=32, g_stride_token=768, g_stride_head=0)), None) == -3


def test_rope_validation_without_touching_cuda():
    """Rotary tables: both or neither, 16-byte aligned rows, head_dim 64 self-attention only; a bad
    combination returns its status before any CUDA call. (Rotary calls need a workspace that also
    holds the rotated q and k.)"""
    base = dict(q=16, k=16, v=16, out=16, cu_seqlens_q=16, cu_seqlens_k=16, workspace=256, workspace_bytes=1 << 40,
                q_stride_token=768, q_stride_head=64, k_stride_token=768, k_stride_head=64, v_stride_token=768,
                v_stride_head=64, o_stride_token=768, o_stride_head=64)
    so = _lib.lib()

    def status(**kw):
        return so.pe_b200_attn_fwd(ctypes.byref(_params(**{**base, **kw})), None)

    assert status(rope_cos=32, rope_stride_token=64) == -1                       # sin missing
    assert status(rope_cos=40, rope_sin=32, rope_stride_token=64) == -3          # misaligned table
    assert status(rope_cos=32, rope_sin=32, rope_stride_token=60) == -3          # rows narrower than D
    assert status(rope_cos=32, rope_sin=32, rope_stride_token=68) == -3          # row stride not 16-byte
    assert status(rope_cos=32, rope_sin=32, rope_stride_token=128, head_dim=128, q_stride_token=1536,
                  q_stride_head=128, k_stride_token=1536, k_stride_head=128, v_stride_token=1536,
                  v_stride_head=128, o_stride_token=1536, o_stride_head=128) == -8  # head_dim 128
    assert status(rope_cos=32, rope_sin=32, rope_stride_token=64, cu_seqlens_k=48) == -8  # other key segments
    assert status(rope_cos=32, rope_sin=32, rope_stride_token=64, total_k=999) == -8      # cross-attention
    need = ctypes.c_size_t(0)
    plain = _params(**base)
    rope = _params(**{**base, "rope_cos": 32, "rope_sin": 32, "rope_stride_token": 64})
    assert so.pe_b200_attn_workspace_size(ctypes.byref(plain), ctypes.byref(need)) == 0
    plain_bytes = need.value
    assert so.pe_b200_attn_workspace_size(ctypes.byref(rope), ctypes.byref(need)) == 0
    assert need.value >= plain_bytes + 2 * 1000 * 12 * 64 * 2  # + rotated q and k
    assert status(rope_cos=32, rope_sin=32, rope_stride_token=64, workspace_bytes=plain_bytes) == -5


def test_rope_pass_validation_without_touching_cuda():
    """pe_b200_rope_qk rejects bad arguments before any CUDA call."""
    so = _lib.lib()

    def status(**kw):
        a = dict(q=16, k=16, qst=2304, qsh=64, kst=2304, ksh=64, cos=32, sin=48, tst=64, rows=100, total=100,
                 heads=12, kv=12, d=64, qo=64, ko=80)
        a.update(kw)
        return so.pe_b200_rope_qk(a["q"], a["k"], a["qst"], a["qsh"], a["kst"], a["ksh"], a["cos"], a["sin"], a["tst"],
                                  a["rows"], a["total"], a["heads"], a["kv"], a["d"], a["qo"], a["ko"], None)

    assert status(d=128) == -8            # head_dim 64 only
    assert status(q=None) == -1           # NULL input
    assert status(cos=40) == -3           # misaligned table
    assert status(qst=2300) == -3         # token stride not a multiple of 16 bytes
    assert status(tst=32) == -3           # table rows narrower than 64
    assert status(rows=0) == -2           # no table rows
    assert status(total=0) == 0           # nothing to do


def test_launch_entry_points_reject_null_workspace_without_touching_cuda():
    p = _params()
    so = _lib.lib()
    assert so.pe_b200_attn_fwd(ctypes.byref(p), None) == -1  # PE_B200_ERR_NULL before any CUDA call


@pytest.mark.parametrize("sym", ["pe_b200_attn_fwd", "pe_b200_build_schedule", "pe_b200_attn_run"])
def test_entry_points_bound(sym):
    assert getattr(_lib.lib(), sym).restype is ctypes.c_int
