"""Host-side wiring of the "b200" backend into the reference package (no GPU needed).

The reference's own tests do the same with monkeypatched loaders
(tests/test_attention_backend.py:29-120): the kernels are replaced by a recorder here.
"""

from __future__ import annotations

import pytest
import torch

from oracle.reference_tree import add_reference_to_path

add_reference_to_path()
pe_ref = pytest.importorskip("packed_encoders")


@pytest.fixture(scope="module")
def installed():
    from packed_encoders_b200 import install

    install.install()
    return install


def test_install_is_idempotent_and_patches_hooks(installed):
    import importlib

    forward = importlib.import_module("packed_encoders.forward")
    ops = importlib.import_module("packed_encoders.ops")
    pack = importlib.import_module("packed_encoders.pack")
    rt = importlib.import_module("packed_encoders.runtime.attention")

    installed.install()
    assert "b200" in rt._CANDIDATES
    assert ops.attention_bshd.__wrapped__ is not None
    assert pack._prepare_modernbert.__wrapped__ is not None
    assert forward.fused_forward.__wrapped__ is not None
    with torch.no_grad():
        assert ops.use_bshd_rope_flash("b200", 12, 64, None)
    assert not ops.use_bshd_rope_flash("b200", 12, 64, None) if torch.is_grad_enabled() else True
    # an unknown backend still behaves as before
    with torch.no_grad():
        assert not ops.use_bshd_rope_flash("sdpa", 12, 64, None)


def test_backend_resolution_keeps_b200(installed):
    from packed_encoders import attention_dispatch, forward

    workload = attention_dispatch.AttentionWorkload.from_lengths([5, 300, 17])
    assert forward._resolve_eager_backend("b200", workload, triton_supported=True, flash_available=True) == "b200"


def _fake_device(monkeypatch, cc, name):
    from packed_encoders import attention_dispatch

    monkeypatch.setattr(attention_dispatch, "current_compute_capability", lambda: cc)
    monkeypatch.setattr(attention_dispatch, "current_device_name", lambda: name)


def test_default_and_auto_resolve_to_b200_on_sm100(installed, monkeypatch):
    """The single b200 backend replaces the calibrated Triton-vs-FA policy on sm_100
    (attention_dispatch.py:129-139 holds the B200 threshold it no longer reaches): the default
    backend of pe.pack (pack.py:147-158), the "auto" branch of pack._resolve_attention_backend
    (pack.py:161-192) and of forward._resolve_eager_backend (forward.py:320-331, eager and
    for_cuda_graph) all give "b200"; the rectangular graph runner is not built for it."""
    import importlib

    from packed_encoders import attention_dispatch, forward, graph

    pack = importlib.import_module("packed_encoders.pack")  # the package re-exports a function of this name
    _fake_device(monkeypatch, (10, 0), "NVIDIA B200")
    consulted = []
    orig_policy = attention_dispatch.get_packed_inference_policy
    monkeypatch.setattr(attention_dispatch, "get_packed_inference_policy",
                        lambda *a, **k: consulted.append(1) or orig_policy(*a, **k))
    workload = attention_dispatch.AttentionWorkload.from_lengths([5, 300, 17])
    with torch.no_grad():
        assert pack._default_backend() == "b200"
        assert pack._resolve_attention_backend("auto") == "b200"
        assert pack._resolve_attention_backend("b200") == "b200"
        for for_graph in (False, True):
            assert forward._resolve_eager_backend("auto", workload, triton_supported=True, flash_available=True,
                                                  for_cuda_graph=for_graph) == "b200"
        # explicit choices are left alone
        assert forward._resolve_eager_backend("sdpa", workload, triton_supported=True, flash_available=True) == "sdpa"
        assert forward._resolve_eager_backend("flash", workload, triton_supported=True, flash_available=True) == "flash"
    assert not consulted
    assert graph.rectangular_graph_backend("b200") is None
    # training keeps the reference's resolution (the kernels are forward-only)
    with torch.enable_grad():
        assert forward._resolve_eager_backend("auto", workload, triton_supported=True, flash_available=True) == "flash"


def test_other_devices_keep_the_reference_policy(installed, monkeypatch):
    import importlib

    from packed_encoders import attention_dispatch, forward

    pack = importlib.import_module("packed_encoders.pack")
    _fake_device(monkeypatch, (9, 0), "NVIDIA H200")
    workload = attention_dispatch.AttentionWorkload.from_lengths([5, 300, 17])
    with torch.no_grad():
        assert pack._resolve_attention_backend("auto") != "b200"
        got = forward._resolve_eager_backend("auto", workload, triton_supported=True, flash_available=True)
        # the H200 policy keeps Triton below 131,073 live tokens (attention_dispatch.py:124-127)
        assert got == "triton"


def test_pack_without_backend_prepares_b200_on_sm100(installed, monkeypatch):
    """pe.pack(model) with no attention_backend on an sm_100 device prepares the b200 state; the
    preparation itself needs no GPU (validation off, the CUDA requirement faked)."""
    import importlib

    pack = importlib.import_module("packed_encoders.pack")
    _fake_device(monkeypatch, (10, 0), "NVIDIA B200")
    monkeypatch.setattr(pack, "_require_cuda", lambda encoder: None)
    from transformers import ModernBertConfig, ModernBertModel

    cfg = ModernBertConfig(vocab_size=512, hidden_size=128, intermediate_size=192, num_hidden_layers=3,
                           num_attention_heads=2, local_attention=128, global_attn_every_n_layers=3,
                           max_position_embeddings=1024, pad_token_id=0)
    model = ModernBertModel(cfg).eval()
    state = pack._prepare_modernbert(model, validate=False)
    assert state.attention_backend == "b200"
    assert state.train_graph_runner is None


def test_train_graph_runner_is_built_on_b200(installed, monkeypatch):
    """pack(..., train_cuda_graph=True) builds the training graph runner with the pack's backend
    (pack.py:216-238); with "b200" the runner's forward calls the b200 attention."""
    import importlib

    pack = importlib.import_module("packed_encoders.pack")
    _fake_device(monkeypatch, (10, 0), "NVIDIA B200")
    monkeypatch.setattr(pack, "_require_cuda", lambda encoder: None)
    from transformers import ModernBertConfig, ModernBertModel

    cfg = ModernBertConfig(vocab_size=512, hidden_size=128, intermediate_size=192, num_hidden_layers=3,
                           num_attention_heads=2, local_attention=128, global_attn_every_n_layers=3,
                           max_position_embeddings=1024, pad_token_id=0)
    model = ModernBertModel(cfg).eval()
    state = pack._prepare_modernbert(model, validate=False, train_cuda_graph=True)
    assert state.attention_backend == "b200"
    assert state.train_graph_runner is not None and state.train_graph_runner._backend == "b200"


def test_candidate_forms_call_the_kernels(installed, monkeypatch):
    from packed_encoders_b200 import ops as b200_ops

    calls = []

    def recorder(q, k, v, cu, max_len, **kw):
        calls.append((cu, max_len, kw))
        return torch.zeros_like(q)

    monkeypatch.setattr(b200_ops, "packed_attention", recorder)
    packed, padded, prefixed = installed.b200_candidate((16, 16), 0.125)
    q = torch.zeros(10, 4, 64)
    k = torch.zeros(10, 2, 64)
    cu = torch.tensor([0, 4, 10], dtype=torch.int32)
    packed(q, k, k, cu, 6, [4, 6], True)
    assert calls[-1][1] == 6 and calls[-1][2]["causal"] and calls[-1][2]["window"] == (16, 16)

    class Static:
        seg_cu32 = torch.tensor([0, 3, 5, 5, 10], dtype=torch.int32)
        seq = 5

    padded(q, k, k, Static, False)
    assert calls[-1][0] is Static.seg_cu32 and calls[-1][1] == 5
    cu_k = torch.tensor([0, 6, 14], dtype=torch.int32)
    prefixed(q, torch.zeros(14, 2, 64), torch.zeros(14, 2, 64), cu, cu_k, 6, 8, [4, 6], [6, 8], True)
    assert calls[-1][2]["cu_seqlens_k"] is cu_k and calls[-1][2]["max_seqlen_k"] == 8


def test_b200_piece_contract(installed):
    from packed_encoders.pieces.attention import BSHD

    piece = installed.b200_attention_bshd_piece()
    assert piece.contract == BSHD
    q = torch.zeros(2, 10, 2, 64)
    piece.check(q, q, q, window=(-1, -1), scaling=0.125, backend="flash")  # rectangular: rows are sequences
    with pytest.raises(Exception):
        piece.check(q, q[:, :5], q, window=(-1, -1), scaling=0.125, backend="flash")
    with pytest.raises(Exception):  # the packed form is one row
        piece.check(q, q, q, window=(-1, -1), scaling=0.125, cu_seqlens=torch.tensor([0, 10], dtype=torch.int32),
                    max_seqlen=10)


def _record_packed(monkeypatch):
    from packed_encoders_b200 import ops as b200_ops

    calls = []

    def recorder(q, k, v, cu, max_len, **kw):
        calls.append((q, cu, max_len, kw))
        return q.clone()

    monkeypatch.setattr(b200_ops, "packed_attention", recorder)
    return calls


def test_attention_leaf_serves_rectangular_b200(installed, monkeypatch):
    """A rectangular [B, H, S, D] call with backend "b200" (the training graph's forward,
    train_graph.py:170-181) runs as B sequences of S tokens: cu_seqlens 0, S, 2S, ..., built on
    the device, and the output comes back as [B, S, H*D] like the reference's flash call."""
    from packed_encoders import ops

    calls = _record_packed(monkeypatch)
    q = torch.randn(3, 2, 10, 64)
    out = ops.attention(q, q, q, mask=None, window=(64, 64), scaling=0.125, backend="b200")
    qf, cu, max_len, kw = calls[-1]
    assert qf.shape == (30, 2, 64) and torch.equal(qf, q.transpose(1, 2).reshape(30, 2, 64))
    assert cu.dtype == torch.int32 and cu.tolist() == [0, 10, 20, 30] and max_len == 10
    assert kw["window"] == (64, 64) and kw["scale"] == 0.125
    assert out.shape == (3, 10, 128) and torch.equal(out, q.transpose(1, 2).reshape(3, 10, 128))


def test_attention_bshd_serves_rectangular_b200(installed, monkeypatch):
    from packed_encoders import ops

    calls = _record_packed(monkeypatch)
    q = torch.randn(2, 7, 2, 64)
    out = ops.attention_bshd(q, q, q, window=(-1, -1), scaling=0.125, backend="b200")
    assert calls[-1][1].tolist() == [0, 7, 14] and calls[-1][2] == 7
    assert out.shape == (2, 7, 128)


def test_pieces_replace_attention_and_rope_slots(installed, monkeypatch):
    """b200_pieces() fills the ModernBERT pieces' BSHD attention and QKV RoPE slots with this
    library's kernels under the reference's contracts (arch/modernbert_pieces.py:24,38;
    pieces/rope.py:97-99); the RoPE piece calls apply_rope_bshd with the reference's arguments."""
    from packed_encoders.pieces.attention import BSHD
    from packed_encoders.pieces.rope import QKV_BSHD

    from packed_encoders_b200 import ops as b200_ops

    pieces = installed.b200_pieces()
    assert pieces.attention_bshd.contract == BSHD and "b200" in pieces.attention_bshd.name
    assert pieces.rope_qkv.contract == QKV_BSHD and "b200" in pieces.rope_qkv.name
    calls = []
    monkeypatch.setattr(b200_ops, "apply_rope_bshd", lambda *a: calls.append(a) or ("q", "k"))
    qkv, cos, sin = torch.zeros(1, 3, 3 * 2 * 64), torch.zeros(3, 64), torch.zeros(3, 64)
    assert pieces.rope_qkv.execute(qkv, 2, 64, cos, sin) == ("q", "k")
    assert calls[-1][1:3] == (2, 64)
