"""LoRA on the MLP projections and configurable target sets (generalising
include/lora.h:22-27, which fixes q/k/v/o) on the GPU against
the fp32 CPU autograd golden (oracle/golden.py, same formula
y += (alpha/r) (x A^T) B^T on gate_proj / up_proj / down_proj).

Same bar as the reference-path step tests: loss 1e-3 relative; every LoRA
gradient and post-AdamW adapter rel-L2 <= 1e-2 and cosine >= 0.999.  Target
subsets leave the other projections at their base weights (no adapter keys
in the golden dict, no parameters in the context)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

LOSS_RTOL = 1e-3
GRAD_RELL2 = 1e-2
GRAD_COS = 0.999
INVALID_ARG = 1


def _ctx(llmcu, cfg, batch, seq, projs, base, lora, int8=False):
    model = llmcu.Model(cfg.hidden, cfg.n_layers, cfg.n_heads, cfg.n_kv_heads, cfg.head_dim, cfg.ffn, cfg.vocab,
                        cfg.rope_theta, cfg.rms_eps)
    run = llmcu.Run(batch, seq, base_dtype=llmcu.BASE_INT8 if int8 else llmcu.BASE_FP16)
    ctx = llmcu.Context(model, llmcu.Lora(cfg.lora_rank, cfg.lora_alpha, llmcu.targets_mask(projs)), run)
    ctx.set_base(base)
    ctx.set_lora_dict(lora)
    return ctx


def _check_dicts(G, got, ref, what):
    assert set(got) == set(ref), (sorted(got), sorted(ref))
    for k in ref:
        r, c = G.rel_l2(got[k], ref[k]), G.cosine(got[k], ref[k])
        assert r <= GRAD_RELL2 and c >= GRAD_COS, f"{what} {k}: rel_l2 {r:.3e} cos {c:.6f}"


def _step_vs_golden(llmcu, G, cfg, batch, seq, seed, projs, golden_base=None, int8=False, threads=None,
                    dist="uniform"):
    base = G.make_base_weights(cfg, seed, round_fp16=True)
    lora = G.make_lora(cfg, seed + 1, projs=projs)
    tok, tgt = G.make_tokens(cfg, batch, seq, seed + 2, dist=dist)
    ctx = _ctx(llmcu, cfg, batch, seq, projs, base, lora, int8=int8)
    assert ctx.lora_param_count() == cfg.n_lora_params(projs)
    assert ctx.lora_targets() == llmcu.targets_mask(projs)
    ref = G.forward_backward(cfg, golden_base(base) if golden_base else base, lora, tok, tgt, threads=threads)
    loss = ctx.forward_backward(tok, tgt)
    assert abs(loss - ref.loss) <= LOSS_RTOL * abs(ref.loss), (loss, ref.loss)
    _check_dicts(G, ctx.grads_dict(), ref.grads, "grad")
    return G, base, lora, ref, ctx


@pytest.mark.parametrize("projs", [
    ("wq", "wk", "wv", "wo", "w_gate", "w_up", "w_down"),
    ("w_gate", "w_up", "w_down"),
    ("wq", "wv", "w_down"),
    ("wk", "w_gate"),
    ("wo", "w_up"),
])
def test_tiny_targets_step_matches_golden(llmcu, cuda_device, projs):
    from oracle import golden as G
    cfg = G.CFG_TINY
    G, base, lora, ref, ctx = _step_vs_golden(llmcu, G, cfg, 2, 64, 31, projs)
    opt = llmcu.AdamW()
    ctx.adamw(opt, step=1)
    upd = {k: a.copy() for k, a in lora.items()}
    G.adamw(upd, ref.grads, G.zeros_like_lora(lora), G.zeros_like_lora(lora), lr=opt.lr, beta1=opt.beta1,
            beta2=opt.beta2, eps=opt.eps, wd=opt.weight_decay, step=1)
    _check_dicts(G, ctx.lora_dict(), upd, "post-adamw")
    # a projection outside the targets has no adapter to set
    missing = [p for p in range(7) if not (ctx.lora_targets() >> p) & 1]
    if missing:
        d_out, d_in = ctx._dims(missing[0])
        with pytest.raises(llmcu.LlmcuError) as e:
            ctx.set_lora(0, missing[0], np.zeros((cfg.lora_rank, d_in), np.float32),
                         np.zeros((d_out, cfg.lora_rank), np.float32))
        assert e.value.status == INVALID_ARG
    ctx.close()


def test_tiny_all_targets_three_steps_track_golden(llmcu, cuda_device):
    from oracle import golden as G
    cfg = G.CFG_TINY
    projs = G.ALL_PROJS
    base = G.make_base_weights(cfg, 41, round_fp16=True)
    lora = G.make_lora(cfg, 42, projs=projs)
    tok, tgt = G.make_tokens(cfg, 1, 48, 43)
    ctx = _ctx(llmcu, cfg, 1, 48, projs, base, lora)
    m, v = G.zeros_like_lora(lora), G.zeros_like_lora(lora)
    ref_lora = {k: a.copy() for k, a in lora.items()}
    opt = llmcu.AdamW()
    for step in range(1, 4):
        r = G.train_step(cfg, base, ref_lora, m, v, tok, tgt, lr=opt.lr, step=step)
        loss = ctx.train_step(tok, tgt, opt, step)
        assert abs(loss - r.loss) <= LOSS_RTOL * abs(r.loss)
    got = ctx.lora_dict()
    _check_dicts(G, got, ref_lora, "3-step adapters")
    for k in lora:
        assert G.cosine(got[k] - lora[k], ref_lora[k] - lora[k]) >= 0.99, k
    ctx.close()


def test_qwen3_shape_slice_all_targets(llmcu, cuda_device):
    """Two layers of the Qwen3-1.7B shape (hd 128, ffn 6144, rank 16: the
    staged dB path and the gate/up interleave at full width), 16384-token
    vocabulary, batch 2 x seq 128, Zipf tokens, every projection adapted."""
    from oracle import golden as G
    cfg = G.layer_slice(G.CFG_QWEN3_1P7B, 2, vocab=16384)
    _, _, _, _, ctx = _step_vs_golden(llmcu, G, cfg, 2, 128, 51, G.ALL_PROJS, threads=8, dist="zipf")
    ctx.close()


def test_int8_base_mlp_targets(llmcu, cuda_device):
    """INT8 base: the MLP's merged weights are built straight from the INT8
    rows and their scales (no per-layer dequantisation)."""
    from oracle import golden as G
    from oracle import quant

    def int8_view(base):
        out = {}
        for k, w in base.items():
            if w.ndim == 2:
                q, s = quant.quantize_rows(w)
                out[k] = (q.astype(np.float32) * s[:, None]).astype(np.float32)
            else:
                out[k] = w
        return out

    cfg = G.CFG_TINY
    _, _, _, _, ctx = _step_vs_golden(llmcu, G, cfg, 2, 64, 61, ("wq", "wo", "w_gate", "w_up", "w_down"),
                                      golden_base=int8_view, int8=True)
    ctx.close()


def test_generate_with_mlp_adapters(llmcu, cuda_device):
    """Greedy decoding reads the merged gate/up and down rows."""
    from oracle import golden as G
    cfg = G.CFG_TINY
    projs = G.ALL_PROJS
    base = G.make_base_weights(cfg, 71, round_fp16=True)
    lora = G.make_lora(cfg, 72, projs=projs, b_std=0.05)
    prompt = G.make_tokens(cfg, 1, 16, 73)[0][0]
    ctx = _ctx(llmcu, cfg, 1, 48, projs, base, lora)
    n_new = 8
    toks, logits, _ = ctx.generate(prompt, n_new, want_logits=True)
    assert np.array_equal(toks, logits.argmax(axis=1).astype(np.int32))
    seq = list(prompt)
    for t in range(n_new):
        ref = G.forward_logits(cfg, base, lora, np.array([seq], dtype=np.int32))[0, -1]
        assert G.rel_l2(logits[t], ref) <= 1e-2, t
        seq.append(int(toks[t]))
    toks2, _, _ = ctx.generate(prompt, n_new)
    assert np.array_equal(toks2, toks)
    ctx.close()


def test_mlp_targets_save_resume_files(llmcu, cuda_device, tmp_path):
    """Adapter files gain the w_gate / w_up / w_down names; the AdamW sidecar
    records the target set and refuses a context with another one."""
    from oracle import golden as G
    cfg = G.CFG_TINY
    projs = ("wq", "wk", "wv", "wo", "w_down")
    base = G.make_base_weights(cfg, 81, round_fp16=True)
    lora = G.make_lora(cfg, 82, projs=projs)
    tok, tgt = G.make_tokens(cfg, 1, 32, 83)
    a = _ctx(llmcu, cfg, 1, 32, projs, base, lora)
    a.train_step(tok, tgt, llmcu.AdamW(), 1)
    a.save_lora(str(tmp_path), 1)
    a.save_adamw_state(str(tmp_path), 1)
    names = sorted(p.name for p in tmp_path.iterdir())
    assert "lora_step1_layer0_w_down_A.bin" in names and "lora_step1_layer1_w_down_B.bin" in names
    assert not any("w_gate" in n or "w_up" in n for n in names)
    b = _ctx(llmcu, cfg, 1, 32, projs, base, G.make_lora(cfg, 99, projs=projs))
    b.load_lora(str(tmp_path), 1)
    b.load_adamw_state(str(tmp_path), 1)
    ga, gb = a.lora_dict(), b.lora_dict()
    for k in ga:
        assert np.array_equal(ga[k], gb[k]), k
    # another target set: the sidecar must refuse it, even at an equal
    # parameter count (w_down and w_up adapters of the tiny shape have the
    # same size)
    for other in (("wq", "wk", "wv", "wo"), ("wq", "wk", "wv", "wo", "w_up")):
        c = _ctx(llmcu, cfg, 1, 32, other, base, G.make_lora(cfg, 84, projs=other))
        with pytest.raises(llmcu.LlmcuError) as e:
            c.load_adamw_state(str(tmp_path), 1)
        assert e.value.status == INVALID_ARG
        c.close()
    for ctx in (a, b):
        ctx.close()
