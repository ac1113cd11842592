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


def test_struct_layout_matches_header():
    # offsets of the C struct on x86-64 (pointers 8, int32 4, int64 8, natural alignment)
    P = _lib.PeB200AttnParams
    assert P.n_seq.offset == 56
    assert P.q_stride_token.offset == 88
    assert P.scale.offset == 152
    assert P.workspace.offset == 168
    assert ctypes.sizeof(P) == 184


def test_launch_entry_points_reject_null_workspace_without_touching_cuda():
    p = _params()
    so = _lib.lib()
    assert so.pe_b200_attn_fwd(ctypes.byref(p), None) == -1  # PE_B200_ERR_NULL before any CUDA call


@pytest.mark.parametrize("sym", ["pe_b200_attn_fwd", "pe_b200_build_schedule", "pe_b200_attn_run"])
def test_entry_points_bound(sym):
    assert getattr(_lib.lib(), sym).restype is ctypes.c_int
