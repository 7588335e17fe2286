"""CPU tests of the oracle (oracle/golden.py, oracle/quant.py): pinned against
the reference's own CUDA trainer (fixtures in tests/golden/, produced by
tests/golden/make_ref_fixtures.py through oracle/ref_harness), plus
known-answer and consistency checks.  No GPU needed."""
import json
import os
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
GOLDEN_DIR = os.path.join(HERE, "golden")
sys.path.insert(0, GOLDEN_DIR)

from oracle import golden as G  # noqa: E402
from oracle.quant import quantize_rows, dequant_gemm_nt  # noqa: E402

with open(os.path.join(GOLDEN_DIR, "ref_tiny_manifest.json")) as _f:
    MANIFEST = json.load(_f)


def _inputs(case):
    import make_ref_fixtures as F
    c = MANIFEST[case]
    return F.case_inputs(G.CFG_TINY, c["batch"], c["seq"], c["seed"], c["dist"])


def _fixture(case):
    z = np.load(os.path.join(GOLDEN_DIR, f"ref_tiny_{case}.npz"))
    grads = {k[5:]: z[k] for k in z.files if k.startswith("grad/")}
    after = {k[6:]: z[k] for k in z.files if k.startswith("after/")}
    return z["losses"], grads, after


@pytest.mark.parametrize("case", sorted(MANIFEST))
def test_golden_with_reference_conventions_matches_reference_build(case):
    """golden(ref_bugs=True) reproduces the reference trainer's loss, LoRA
    gradients and post-AdamW adapters (fp32 vs fp32: only summation order and
    libm differ)."""
    base, lora, tok, tgt = _inputs(case)
    losses, grads, after = _fixture(case)
    res = G.forward_backward(G.CFG_TINY, base, lora, tok, tgt, ref_bugs=True)
    assert abs(res.loss - float(np.mean(losses))) <= 1e-5 * abs(res.loss)
    for k in grads:
        assert G.rel_l2(res.grads[k], grads[k]) <= 1e-4, k
    upd = {k: a.copy() for k, a in lora.items()}
    lr, b1, b2, eps, wd = MANIFEST[case]["adamw"]
    G.adamw(upd, res.grads, G.zeros_like_lora(lora), G.zeros_like_lora(lora), lr=lr, beta1=b1, beta2=b2, eps=eps,
            wd=wd, step=1)
    for k in after:
        assert G.rel_l2(upd[k], after[k]) <= 1e-5, k


@pytest.mark.parametrize("case", sorted(MANIFEST))
def test_true_gradient_golden_shares_the_reference_forward(case):
    """The default (true-gradient) golden has the same forward/loss as the
    reference build; its gradients differ only through the four documented
    deviations of the reference's hand-written backward."""
    base, lora, tok, tgt = _inputs(case)
    losses, grads, _ = _fixture(case)
    res = G.forward_backward(G.CFG_TINY, base, lora, tok, tgt)
    assert abs(res.loss - float(np.mean(losses))) <= 1e-5 * abs(res.loss)
    # with B != 0 (configs[0] init) the reference's misread-A dX term changes every layer's gradient
    assert max(G.rel_l2(res.grads[k], grads[k]) for k in grads) > 1e-2


def test_ref_bug_switches_are_the_only_difference():
    """With B = 0 (the reference's own adapter init) the misread-A dX term vanishes
    and both goldens share the forward; dA is exactly zero in both."""
    cfg = G.CFG_TINY
    base = G.make_base_weights(cfg, 1)
    lora = G.make_lora(cfg, 2, b_std=0.0)
    tok, tgt = G.make_tokens(cfg, 1, 16, 3)
    a = G.forward_backward(cfg, base, lora, tok, tgt)
    b = G.forward_backward(cfg, base, lora, tok, tgt, ref_bugs=True)
    assert a.loss == pytest.approx(b.loss, rel=1e-7)
    # B = 0: dA is exactly zero in both (dh = dy . B = 0)
    for k in a.grads:
        if k.endswith(".A"):
            assert np.all(a.grads[k] == 0) and np.all(b.grads[k] == 0)


def test_golden_gradient_matches_finite_differences():
    """Autograd of the golden against a central difference of its own loss on
    a few adapter entries of every projection kind, MLP adapters included
    (float64 tiny model)."""
    import torch
    torch.set_default_dtype(torch.float64)
    try:
        cfg = G.ModelCfg(hidden=64, n_layers=1, n_heads=2, n_kv_heads=1, head_dim=64, ffn=128, vocab=97,
                         lora_rank=2, lora_alpha=4.0)
        base = {k: v.astype(np.float64) for k, v in G.make_base_weights(cfg, 5, std=0.2).items()}
        lora = {k: v.astype(np.float64) for k, v in G.make_lora(cfg, 6, b_std=0.2, projs=G.ALL_PROJS).items()}
        tok, tgt = G.make_tokens(cfg, 1, 8, 7)
        res = G.forward_backward(cfg, base, lora, tok, tgt)
        rng = np.random.default_rng(0)
        for key in ("L0.wq.A", "L0.wv.B", "L0.wo.A", "L0.wk.B", "L0.w_gate.A", "L0.w_up.B", "L0.w_down.A",
                    "L0.w_down.B"):
            idx = tuple(rng.integers(0, s) for s in lora[key].shape)
            h = 1e-5
            lp = {k: v.copy() for k, v in lora.items()}
            lm = {k: v.copy() for k, v in lora.items()}
            lp[key][idx] += h
            lm[key][idx] -= h
            fd = (G.forward_backward(cfg, base, lp, tok, tgt).loss - G.forward_backward(cfg, base, lm, tok, tgt).loss) / (2 * h)
            assert res.grads[key][idx] == pytest.approx(fd, rel=1e-4, abs=1e-9), key
    finally:
        torch.set_default_dtype(torch.float32)


def test_loss_conventions():
    cfg = G.CFG_TINY
    base = G.make_base_weights(cfg, 1)
    lora = G.make_lora(cfg, 2)
    tok, tgt = G.make_tokens(cfg, 2, 16, 3)
    a = G.forward_backward(cfg, base, lora, tok, tgt)
    b = G.forward_backward(cfg, base, lora, tok, tgt, all_positions=True)
    assert a.n_positions == 2 * 15 and b.n_positions == 2 * 16
    # near-uniform random model: the loss is close to ln(V)
    assert abs(a.loss - np.log(cfg.vocab)) < 0.5


def test_flop_model_per_token_figures():
    f = G.algorithmic_flops_per_token(G.CFG_QWEN3_1P7B, 512)
    assert f / 1e9 == pytest.approx(7.097, abs=2e-3)
    assert G.algorithmic_flops_per_token(G.CFG_QWEN3_1P7B, 4096) / 1e9 == pytest.approx(8.330, abs=2e-3)
    assert G.CFG_QWEN3_1P7B.n_lora_params() == 6422528
    assert G.CFG_TINY.n_lora_params() == 14336


# --------------------------------------------------------------- INT8 quantiser

def test_quantiser_known_answers():
    """Hand-computed rows: scale = absmax/127, q = rint(w * (1/scale))."""
    w = np.array([[0.0, 0.0, 0.0],                   # zero row: scale 0, q 0
                  [1.27, -1.27, 0.635],              # absmax 1.27 -> scale 0.01
                  [2.0, 1.0, -0.5],                  # -> 127, 63.5 -> 64 (ties to even), -31.75 -> -32
                  [-3.0, 0.0, 3.0]], np.float32)
    q, s = quantize_rows(w)
    assert s[0] == 0 and np.all(q[0] == 0)
    assert s[1] == np.float32(1.27) / np.float32(127)
    assert q[1].tolist() == [127, -127, 64]
    assert q[2].tolist() == [127, 64, -32]
    assert q[3].tolist() == [-127, 0, 127]
    assert q.dtype == np.int8 and s.dtype == np.float32


def test_quantiser_is_the_fp32_operation_sequence():
    """Every element equals rint(clamp(fl(w * fl(1 / fl(absmax / 127))))) and
    |q| <= 127; dequantised rows are within half a step of the input."""
    rng = np.random.Generator(np.random.PCG64(3))
    w = (rng.standard_normal((64, 333), dtype=np.float32) * np.float32(0.02)).astype(np.float16).astype(np.float32)
    q, s = quantize_rows(w)
    for r in range(w.shape[0]):
        sc = np.float32(np.max(np.abs(w[r]))) / np.float32(127.0)
        inv = np.float32(1.0) / sc
        expect = np.rint(np.clip(w[r] * inv, -127, 127)).astype(np.int8)
        assert np.array_equal(q[r], expect)
        assert np.all(np.abs(q[r].astype(np.float64) * sc - w[r]) <= (0.5 + 1e-4) * sc)
    assert np.abs(q.astype(np.int32)).max() == 127


def test_dequant_gemm_restatement():
    rng = np.random.Generator(np.random.PCG64(4))
    w = rng.standard_normal((16, 32), dtype=np.float32)
    a = rng.standard_normal((5, 32), dtype=np.float32)
    q, s = quantize_rows(w)
    c = dequant_gemm_nt(a, q, s)
    ref = a.astype(np.float64) @ (q.astype(np.float64) * s[:, None].astype(np.float64)).T
    np.testing.assert_allclose(c, ref, rtol=1e-5, atol=1e-5)


def test_golden_mlp_adapters_equal_merged_base():
    """The golden's LoRA terms on gate/up/down are the rank-r update of the
    base weight: forward logits with adapters equal those of the base with
    W + s B A folded in and no adapters on those projections."""
    cfg = G.CFG_TINY
    base = G.make_base_weights(cfg, 3)
    lora = G.make_lora(cfg, 4, projs=G.ALL_PROJS, b_std=0.05)
    tok, _ = G.make_tokens(cfg, 2, 24, 5)
    got = G.forward_logits(cfg, base, lora, tok)
    merged = {k: v.copy() for k, v in base.items()}
    attn_only = {}
    for k, v in lora.items():
        l, p, ab = k.split(".")
        if p in G.MLP_PROJS:
            if ab == "A":
                w = f"{l}.{p}"
                merged[w] = merged[w] + cfg.lora_scale * (lora[f"{l}.{p}.B"] @ lora[f"{l}.{p}.A"])
        else:
            attn_only[k] = v
    ref = G.forward_logits(cfg, merged, attn_only, tok)
    assert G.rel_l2(got, ref) < 1e-5
    # and the MLP terms are not empty
    plain = G.forward_logits(cfg, base, attn_only, tok)
    assert G.rel_l2(got, plain) > 1e-3


def test_golden_target_subsets():
    cfg = G.CFG_QWEN3_1P7B
    assert cfg.n_lora_params() == 6_422_528                      # the reference's q/k/v/o
    assert cfg.n_lora_params(G.MLP_PROJS) == 28 * 3 * 16 * (2048 + 6144)
    tiny = G.CFG_TINY
    lora = G.make_lora(tiny, 1, projs=("wk", "w_down"))
    assert sorted({k.split(".")[1] for k in lora}) == ["w_down", "wk"]
    assert lora["L0.w_down.A"].shape == (4, 768) and lora["L0.w_down.B"].shape == (256, 4)
    # gradients exist exactly for the adapters present
    base = G.make_base_weights(tiny, 2)
    tok, tgt = G.make_tokens(tiny, 1, 16, 3)
    res = G.forward_backward(tiny, base, lora, tok, tgt)
    assert set(res.grads) == set(lora)
    assert all(np.abs(g).sum() > 0 for g in res.grads.values())


def test_bench_flop_model_and_targets():
    """bench.py's own FLOP model (no oracle import on its timed path) equals the
    golden's, for the reference's targets and for all seven; its --lora-targets
    parser keeps the projection order and rejects unknown names."""
    import importlib.util
    spec = importlib.util.spec_from_file_location("bench_mod", os.path.join(os.path.dirname(HERE), "bench.py"))
    b = importlib.util.module_from_spec(spec)
    sys.modules["bench_mod"] = b
    spec.loader.exec_module(b)
    from conftest import load_binding
    m = load_binding()
    model = m.Model.qwen3_1p7b()
    full = G.CFG_QWEN3_1P7B
    for projs in (G.PROJS, G.ALL_PROJS):
        got = b.algorithmic_flops_per_token(model, 512, full.n_lora_params(projs))
        assert got == pytest.approx(G.algorithmic_flops_per_token(full, 512, projs), rel=1e-12)
    assert b.parse_targets("attn") == G.PROJS
    assert b.parse_targets("all") == G.ALL_PROJS
    assert b.parse_targets("w_down,wq") == ("wq", "w_down")
    with pytest.raises(SystemExit):
        b.parse_targets("wq,w_bogus")
