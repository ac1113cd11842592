"""The "b200" backend driven by the reference's own entry points (GPU).

The reference package is imported from its git-ignored install in baseline/_ref; the tests
skip when it is absent. They mirror the
reference's own GPU tests:

* packed vs stock HF ModernBERT on padded batches, per-token cosine > 0.997
  (tests/test_varlen.py:165-187), here with a small random-init model;
* ``packed_forward`` on b200 vs the reference's dependency-free SDPA backend;
* ``runtime.attention.select_attention`` probing the b200 candidate for the Qwen3.5 GQA
  geometry 8/2/256, causal and bidirectional, including the prefixed form
  (tests/test_qwen35.py:136-152), and a windowed scale-bound kind
  (tests/test_embedding_gemma2.py:106-115).
"""

from __future__ import annotations

import copy

import pytest
import torch
import torch.nn.functional as F

from oracle.reference_tree import add_reference_to_path

add_reference_to_path()

pytestmark = pytest.mark.gpu
pe_ref = pytest.importorskip("packed_encoders")


@pytest.fixture(scope="module")
def b200():
    from packed_encoders_b200 import install

    install.install()
    return install


def _tiny_modernbert(seed=0, layers=3):
    from transformers import ModernBertConfig, ModernBertModel

    torch.manual_seed(seed)
    cfg = ModernBertConfig(vocab_size=512, hidden_size=128, intermediate_size=192, num_hidden_layers=layers,
                           num_attention_heads=2, local_attention=128, global_attn_every_n_layers=3,
                           max_position_embeddings=1024, pad_token_id=0)
    cfg._attn_implementation = "sdpa"
    model = ModernBertModel(cfg).to("cuda", torch.bfloat16).eval()
    return model


def _masked_cos(out, ref, am):
    m = am.bool().unsqueeze(-1).expand_as(ref)
    return F.cosine_similarity(out[m].float(), ref[m].float(), dim=0).item()


def _per_token_min_cos(out, ref, am):
    keep = am.bool()
    return F.cosine_similarity(out[keep].float(), ref[keep].float(), dim=-1).min().item()


def test_pack_b200_matches_stock_hf_on_padded_batch(b200):
    from packed_encoders.arch.modernbert import ModernBert

    stock = _tiny_modernbert()
    packed = copy.deepcopy(stock)
    # validate=False: the reference's validation gate refuses this image's nvidia-cutlass-dsl 4.5.0
    # (its floor is 4.5.2, validate.py:80-110); the comparison with stock HF below is the check.
    pe_ref.pack(packed, engine=ModernBert(pieces=b200.b200_pieces()), attention_backend="b200", validate=False)
    lengths = [7, 300, 1, 129, 200]
    s = max(lengths)
    gen = torch.Generator(device="cuda").manual_seed(1)
    ids = torch.randint(1, 512, (len(lengths), s), device="cuda", generator=gen)
    am = torch.zeros_like(ids)
    for i, n in enumerate(lengths):
        am[i, :n] = 1
    ids = ids * am
    with torch.inference_mode():
        ref = stock(input_ids=ids, attention_mask=am).last_hidden_state
        out = packed(input_ids=ids, attention_mask=am).last_hidden_state
    assert torch.isfinite(out[am.bool()]).all()
    assert _masked_cos(out, ref, am) > 0.997
    assert _per_token_min_cos(out, ref, am) > 0.98


def test_pack_with_default_backend_runs_b200_kernels(b200):
    """pe.pack(model) with no attention_backend on an sm_100 GPU resolves to "b200" (the
    calibrated Triton-vs-FA policy is replaced, attention_dispatch.py:129-139) and the forward
    launches this library's kernels; outputs match stock HF."""
    from packed_encoders_b200 import ops as b200_ops

    if torch.cuda.get_device_capability() != (10, 0):
        pytest.skip("the b200 default applies to sm_100 devices")
    stock = _tiny_modernbert(seed=4)
    packed = copy.deepcopy(stock)
    pe_ref.pack(packed, validate=False)
    from packed_encoders.state import ATTR

    assert getattr(packed, ATTR).attention_backend == "b200"
    lengths = [9, 200, 1, 64]
    s = max(lengths)
    gen = torch.Generator(device="cuda").manual_seed(2)
    ids = torch.randint(1, 512, (len(lengths), s), device="cuda", generator=gen)
    am = torch.zeros_like(ids)
    for i, n in enumerate(lengths):
        am[i, :n] = 1
    ids = ids * am
    before = b200_ops.LAUNCHES["kernels"]
    with torch.inference_mode():
        out = packed(input_ids=ids, attention_mask=am).last_hidden_state
        ref = stock(input_ids=ids, attention_mask=am).last_hidden_state
    assert b200_ops.LAUNCHES["kernels"] > before
    assert _masked_cos(out, ref, am) > 0.997


def test_packed_forward_b200_matches_reference_sdpa_backend(b200):
    from packed_encoders import forward
    from packed_encoders.arch.modernbert import ModernBert
    from packed_encoders.config import ModernBertParams

    model = _tiny_modernbert(seed=2)
    pe_ref.pack(model, engine=ModernBert(pieces=b200.b200_pieces()), attention_backend="b200", validate=False)
    params = ModernBertParams.from_hf_config(model.config)
    lengths = [5, 140, 33, 260]
    cu = torch.tensor([0, *torch.tensor(lengths).cumsum(0).tolist()], dtype=torch.int32, device="cuda")
    gen = torch.Generator(device="cuda").manual_seed(3)
    ids = torch.randint(1, 512, (sum(lengths),), device="cuda", generator=gen)
    pos = torch.cat([torch.arange(n, device="cuda") for n in lengths])
    with torch.inference_mode():
        out = forward.packed_forward(model, params, ids, cu, max(lengths), pos, backend="b200")
        ref = forward.packed_forward(model, params, ids, cu, max(lengths), pos, backend="sdpa")
    cos = F.cosine_similarity(out.float(), ref.float(), dim=-1)
    assert cos.mean().item() > 0.999 and cos.min().item() > 0.99


@pytest.mark.parametrize("causal", [False, True])
def test_select_attention_accepts_b200_for_qwen_geometry(b200, causal):
    from packed_encoders.runtime.attention import PROBE_TOLERANCE, select_attention

    choice = select_attention(n_heads=8, n_kv_heads=2, head_dim=256, causal=causal, device=torch.device("cuda"),
                              order=("b200",))
    assert choice.name == "b200", choice.rejected
    assert choice.max_abs_err < PROBE_TOLERANCE
    assert (choice.prefixed is not None) == causal
    if causal:
        assert choice.prefixed_name == "b200" and choice.prefixed_max_abs_err < PROBE_TOLERANCE


def test_select_attention_b200_windowed_kind(b200):
    from packed_encoders.runtime.attention import PROBE_TOLERANCE, select_attention

    choice = select_attention(n_heads=4, n_kv_heads=1, head_dim=64, causal=False, device=torch.device("cuda"),
                              order=("b200",), window=(16, 16), scale=0.125)
    assert choice.name == "b200", choice.rejected
    assert choice.max_abs_err < PROBE_TOLERANCE


def test_default_order_prefers_b200_on_sm100(b200):
    from packed_encoders.runtime.attention import default_order

    if torch.cuda.get_device_capability() == (10, 0):
        assert default_order(torch.device("cuda"))[0] == "b200"


def test_apply_rope_bshd_matches_reference_kernel(b200):
    """This library's RoPE pass against the reference's own apply_rope_bshd (CuteDSL,
    _kernels/rope.py:302-345) on the same packed qkv and per-token tables: same shapes, and the
    same bf16 values up to rare last-bit differences of the fp32 rotation's rounding."""
    import packed_encoders_b200 as pe

    try:
        from packed_encoders._kernels.rope import apply_rope_bshd as ref_rope
    except Exception as exc:  # noqa: BLE001
        pytest.skip(f"reference rope kernel unavailable: {type(exc).__name__}")
    heads, d, total = 12, 64, 1537
    gen = torch.Generator(device="cuda").manual_seed(5)
    qkv = torch.randn(1, total, 3 * heads * d, device="cuda", generator=gen).to(torch.bfloat16)
    pos = torch.arange(total, device="cuda", dtype=torch.float32) % 700
    inv = 1.0 / 10000.0 ** (torch.arange(0, d, 2, device="cuda", dtype=torch.float32) / d)
    emb = torch.cat((pos[:, None] * inv, pos[:, None] * inv), -1)
    cos, sin = emb.cos().to(torch.bfloat16), emb.sin().to(torch.bfloat16)
    q, k = pe.apply_rope_bshd(qkv, heads, d, cos, sin)
    rq, rk = ref_rope(qkv, heads, d, cos, sin)
    assert q.shape == rq.shape and k.shape == rk.shape
    for a, b in ((q, rq), (k, rk)):
        assert (a.float() - b.float()).abs().max().item() <= 2.0 ** -6 * b.float().abs().max().item()
        assert (a != b).float().mean().item() < 0.01



@pytest.mark.parametrize("gated", [False, True])
def test_qwen35_attention_caller_runs_b200(b200, gated):
    """The Qwen3.5 engine's attention path (arch/qwen3_5/engine.py:551-571 -> execution.py:24-27):
    OrdinaryExecution.attention calls the engine's bound attention_packed piece with the
    runtime choice, here the b200 candidate selected for the 8/2/256 causal geometry, and the
    gated layers apply the engine's sigmoid_gate piece after it. Checked against the oracle (plus
    the reference's gate roundings) and, for the gated form, against this library's own gate
    in the attention call (same bits)."""
    from types import SimpleNamespace

    import oracle
    from conftest import packed_inputs
    from packed_encoders.arch.qwen3_5.execution import OrdinaryExecution
    from packed_encoders.arch.qwen3_5.pieces import default_pieces
    from packed_encoders.runtime.attention import select_attention

    import packed_encoders_b200 as pe

    choice = select_attention(n_heads=8, n_kv_heads=2, head_dim=256, causal=True, device=torch.device("cuda"),
                              order=("b200",))
    assert choice.name == "b200", choice.rejected
    engine = SimpleNamespace(ops=default_pieces().bind(), attention=choice, causal=True)
    lengths = [300, 5, 1000, 64, 129]
    q, k, v, cu = packed_inputs(lengths, 8, 256, kv_heads=2, seed=61)
    lay = SimpleNamespace(static=None, cu32=cu.cuda(), max_len=max(lengths), lengths=lengths)
    before = pe.ops.LAUNCHES["kernels"]
    with torch.inference_mode():
        o = OrdinaryExecution.attention(engine, q.cuda(), k.cuda(), v.cuda(), lay)
    torch.cuda.synchronize()
    assert pe.ops.LAUNCHES["kernels"] > before
    ref, _ = oracle.attention(q, k, v, cu, scale=256 ** -0.5, causal=True)
    err = (o.float().cpu() - ref).abs().max().item()
    print(f"PARITY qwen35 caller: max_abs={err:.5f}")
    assert err <= 2e-2
    if gated:
        gate = (torch.randn(q.shape, generator=torch.Generator().manual_seed(62)) * 2).to(torch.bfloat16).cuda()
        with torch.inference_mode():
            y = engine.ops.sigmoid_gate(o.view(o.shape[0], 8, 256), gate)
            fused = pe.packed_attention(q.cuda(), k.cuda(), v.cuda(), cu.cuda(), max(lengths), scale=256 ** -0.5,
                                        causal=True, gate=gate)
        torch.cuda.synchronize()
        ref_y = (ref.to(torch.bfloat16).float() * torch.sigmoid(gate.float().cpu()).to(torch.bfloat16).float())
        gerr = (y.float().cpu().view_as(ref_y) - ref_y).abs().max().item()
        print(f"PARITY qwen35 gated caller: max_abs={gerr:.5f}")
        assert gerr <= 2e-2
        # same roundings; a sigmoid within an ulp of a bf16 rounding boundary may round the other way
        diff = (fused.view(fused.shape[0], -1).float() - y.float()).abs()
        assert (diff > 0).float().mean().item() < 0.01 and diff.max().item() <= 2e-2


# --------------------------------------------------------------------------- training
def _grads_of_interest(model):
    """The output-proximate parameter gradients the reference's training test compares
    (tests/test_varlen.py:250-268): the final norm and, in the last three layers, Wqkv, Wo, Wi, the
    MLP's Wo and the MLP norm."""
    picks = {"final_norm": model.final_norm.weight}
    n = len(model.layers)
    for li in (n - 1, n - 2, n - 3):
        layer = model.layers[li]
        picks[f"L{li}.attn.Wqkv"] = layer.attn.Wqkv.weight
        picks[f"L{li}.attn.Wo"] = layer.attn.Wo.weight
        picks[f"L{li}.mlp.Wi"] = layer.mlp.Wi.weight
        picks[f"L{li}.mlp.Wo"] = layer.mlp.Wo.weight
        picks[f"L{li}.mlp_norm"] = layer.mlp_norm.weight
    return {name: p.grad.detach().float().clone() for name, p in picks.items()}


def _train_step_grads(model, ids, am, seed):
    """One forward + backward of the real tokens' outputs projected on a fixed random tensor. (The
    reference's test squares the outputs, tests/test_varlen.py:271-282; after the final LayerNorm of
    a random-init model that loss is almost constant, and its gradients are bf16 rounding noise.)"""
    model.zero_grad(set_to_none=True)
    out = model(input_ids=ids, attention_mask=am).last_hidden_state
    loss = (out.float() * seed * am.unsqueeze(-1)).sum()
    loss.backward()
    return _grads_of_interest(model)


def _grad_cos(a, b):
    return F.cosine_similarity(a.flatten(), b.flatten(), dim=0).item()


def test_packed_training_step_on_b200_matches_sdpa_and_hf(b200, monkeypatch):
    """A training step of a model packed with "b200" on a padded batch: the grad-enabled forward
    takes the packed path (forward.py:634-657), each layer's attention runs this library's forward
    kernel and its backward kernel (one backward call per layer), and the output-proximate
    gradients are as close to stock HF run in fp32 (the same weights, upcast) as the reference's own
    bf16 paths are (its SDPA backend and stock HF in bf16; the reference's test compares the packed
    gradients with those two at cosine > 0.998, tests/test_varlen.py:304-348): no more than 0.002
    below the closer of the two, and above 0.998 against the SDPA backend."""
    from packed_encoders import forward
    from packed_encoders_b200 import ops as b200_ops

    stock = _tiny_modernbert(seed=5, layers=6)
    on_b200, on_sdpa = copy.deepcopy(stock), copy.deepcopy(stock)
    pe_ref.pack(on_b200, attention_backend="b200", validate=False)
    pe_ref.pack(on_sdpa, attention_backend="sdpa", validate=False)
    lengths = [40, 300, 7, 129, 220]
    gen = torch.Generator(device="cuda").manual_seed(11)
    ids = torch.randint(1, 512, (len(lengths), max(lengths)), device="cuda", generator=gen)
    am = torch.zeros_like(ids)
    for i, n in enumerate(lengths):
        am[i, :n] = 1
    ids = ids * am
    seed = torch.randn(*ids.shape, stock.config.hidden_size, device="cuda", generator=gen)

    calls = {"varlen": 0, "backward": 0}
    orig_varlen, orig_bwd = forward._varlen_forward, b200_ops.packed_attention_backward

    def varlen_spy(*a, **k):
        calls["varlen"] += 1
        return orig_varlen(*a, **k)

    def bwd_spy(*a, **k):
        calls["backward"] += 1
        return orig_bwd(*a, **k)

    monkeypatch.setattr(forward, "_varlen_forward", varlen_spy)
    monkeypatch.setattr(b200_ops, "packed_attention_backward", bwd_spy)
    g_b200 = _train_step_grads(on_b200, ids, am, seed)
    assert calls == {"varlen": 1, "backward": len(stock.layers)}
    g_sdpa = _train_step_grads(on_sdpa, ids, am, seed)
    g_hf = _train_step_grads(stock, ids, am, seed)
    g_fp32 = _train_step_grads(copy.deepcopy(stock).float(), ids, am, seed)
    cos = {name: tuple(round(_grad_cos(g[name], g_fp32[name]), 6) for g in (g_b200, g_sdpa, g_hf))
           + (round(_grad_cos(g_b200[name], g_sdpa[name]), 6),) for name in g_b200}
    print("packed training grads, cosine to fp32 HF of b200 / reference sdpa / HF bf16, and b200-vs-sdpa: "
          f"{cos}")
    for name, (c_b200, c_sdpa, c_hf, c_pair) in cos.items():
        assert c_b200 >= max(c_sdpa, c_hf) - 0.002, f"{name}: b200 {c_b200:.5f} vs sdpa {c_sdpa:.5f} / HF {c_hf:.5f}"
        assert c_pair > 0.998, f"{name}: b200 vs sdpa {c_pair:.5f}"


def _flat_grads(weights):
    return torch.cat([p.grad.float().flatten() for p in weights])


def test_training_graph_on_b200_matches_eager_dense(b200):
    """The reference's training-graph runner (train_graph.py:118-293) built with backend "b200":
    the captured forward calls the rectangular b200 attention (each row one sequence, the window
    per layer), the captured backward replays this library's backward kernels, and the gradients
    match the eager dense SDPA forward it stands in for (the reference test's bars: cosine > 0.999,
    relative L2 < 2e-2, tests/test_train_graph.py:122-142). pack(train_cuda_graph=True) routes the
    grad-enabled forward through that runner."""
    from packed_encoders import forward
    from packed_encoders.config import ModernBertParams
    from packed_encoders.state import get_state
    from packed_encoders_b200 import ops as b200_ops

    model = _tiny_modernbert(seed=6)
    params = ModernBertParams.from_hf_config(model.config)
    weights = [p for p in model.parameters() if p.requires_grad]
    for p in weights:
        p.grad = torch.zeros_like(p)
    pe_ref.pack(model, attention_backend="b200", train_cuda_graph=True, cuda_graph_seq_cutoff=256, validate=False)
    runner = get_state(model).train_graph_runner
    assert runner is not None and runner._backend == "b200"
    b, s = 8, 192
    gen = torch.Generator(device="cuda").manual_seed(12)
    ids = torch.randint(5, 512, (b, s), device="cuda", generator=gen)
    mask = torch.ones((b, s), dtype=torch.long, device="cuda")
    grad_seed = torch.randn((b, s, model.config.hidden_size), device="cuda", generator=gen, dtype=torch.bfloat16)

    before = b200_ops.LAUNCHES["kernels"]
    for p in weights:
        p.grad.zero_()
    out = model(input_ids=ids, attention_mask=mask).last_hidden_state
    out.backward(grad_seed)
    g_graph = _flat_grads(weights)
    assert len(runner._cache) == 1 and b200_ops.LAUNCHES["kernels"] > before

    p = forward.prologue(model, params, ids, mask, dense_mask=True, capture_safe=True)
    ref = forward.core(model, params, p.x, p.cos_global, p.sin_global, p.cos_local, p.sin_local, p.full_mask,
                       p.sliding_mask, backend="sdpa")
    grads = torch.autograd.grad(ref, weights, grad_seed, allow_unused=True)
    g_eager = torch.cat([(g if g is not None else torch.zeros_like(w)).float().flatten()
                         for g, w in zip(grads, weights)])
    cos = _grad_cos(g_graph, g_eager)
    rel = ((g_graph - g_eager).norm() / (g_eager.norm() + 1e-9)).item()
    fwd_cos = _grad_cos(out.detach().float(), ref.detach().float())
    print(f"training graph on b200: forward cosine {fwd_cos:.6f}, grad cosine {cos:.6f}, grad rel L2 {rel:.4f}")
    assert fwd_cos > 0.99 and cos > 0.999 and rel < 2e-2
