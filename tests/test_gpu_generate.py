"""KV-cache generation on the GPU (inference reuse of the training context's
weights and current adapters, as llm_engine --generate does with its own,
src/main.cu:340-385) against the fp32 CPU golden.

Every step's logits must match the golden's logits of the same prefix to
rel-L2 <= 1e-2 (fp16 activations against fp32), the chosen ids must be the
argmax of those logits, and they must equal the golden's greedy ids for as
long as the golden's top-two margin leaves no room for an fp16 tie.  The
graph-replayed decode (no logits requested) must choose the same ids."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

LOGIT_RELL2 = 1e-2


def _ctx(llmcu, G, cfg, base, lora, max_seq, int8=False):
    model = llmcu.Model(cfg.hidden, cfg.n_layers, cfg.n_heads, cfg.n_kv_heads, cfg.head_dim, cfg.ffn, cfg.vocab,
                        cfg.rope_theta, cfg.rms_eps)
    run = llmcu.Run(1, max_seq, base_dtype=llmcu.BASE_INT8) if int8 else llmcu.Run(1, max_seq)
    ctx = llmcu.Context(model, llmcu.Lora(cfg.lora_rank, cfg.lora_alpha), run)
    ctx.set_base(base)
    ctx.set_lora_dict(lora)
    return ctx


def _check(G, cfg, ctx, golden_base, lora, prompt, n_new):
    toks, logits, _ = ctx.generate(prompt, n_new, want_logits=True)
    assert toks.shape == (n_new,)  # no end ids in these vocabularies
    assert np.array_equal(toks, logits.argmax(axis=1).astype(np.int32))
    seq = list(prompt)
    for t in range(n_new):
        ref = G.forward_logits(cfg, golden_base, lora, np.array([seq], dtype=np.int32))[0, -1]
        r = G.rel_l2(logits[t], ref)
        assert r <= LOGIT_RELL2, (t, r)
        top2 = np.sort(ref)[-2:]
        if top2[1] - top2[0] < 2e-2 * np.abs(ref).max():
            break  # a near tie: the continuations may part here
        assert toks[t] == int(np.argmax(ref)), (t, toks[t], int(np.argmax(ref)))
        seq.append(int(toks[t]))
    # the CUDA-graph decode path picks the same ids
    toks2, _, ms = ctx.generate(prompt, n_new)
    assert np.array_equal(toks2, toks)
    assert ms > 0.0
    return toks


def test_generate_tiny_matches_golden(llmcu, cuda_device):
    from oracle import golden as G
    cfg = G.CFG_TINY
    base = G.make_base_weights(cfg, 61, round_fp16=True)
    lora = G.make_lora(cfg, 62)
    prompt = G.make_tokens(cfg, 1, 12, 63)[0][0]
    ctx = _ctx(llmcu, G, cfg, base, lora, max_seq=64)
    _check(G, cfg, ctx, base, lora, prompt, 10)
    # a second call reuses the captured decode graph; a longer prompt
    prompt2 = G.make_tokens(cfg, 1, 40, 64)[0][0]
    _check(G, cfg, ctx, base, lora, prompt2, 6)
    # after a training step the generation uses the updated adapters
    tok, tgt = G.make_tokens(cfg, 1, 32, 65)
    ctx.train_step(tok, tgt, llmcu.AdamW(), 1)
    _check(G, cfg, ctx, base, ctx.lora_dict(), prompt, 6)
    ctx.close()


def test_generate_1p7b_slice_matches_golden(llmcu, cuda_device):
    """head_dim 128, 16 / 8 heads, ffn 6144: the shapes of the production decode kernels."""
    from oracle import golden as G
    cfg = G.layer_slice(G.CFG_QWEN3_1P7B, 2, vocab=16384)
    base = G.make_base_weights(cfg, 71, round_fp16=True)
    lora = G.make_lora(cfg, 72)
    prompt = G.make_tokens(cfg, 1, 20, 73, dist="zipf")[0][0]
    ctx = _ctx(llmcu, G, cfg, base, lora, max_seq=300)
    _check(G, cfg, ctx, base, lora, prompt, 5)
    ctx.close()


def _int8_view(base):
    """The weights the INT8 path computes with: linear weights (and the tied
    embedding) quantised per output row and dequantised in fp32."""
    from oracle import quant
    out = {}
    for k, w in base.items():
        if w.ndim == 2:
            q, s = quant.quantize_rows(w)
            out[k] = (q.astype(np.float32) * s[:, None]).astype(np.float32)
        else:
            out[k] = w
    return out


def test_generate_int8_base_matches_golden(llmcu, cuda_device):
    """INT8 base: the MLP and lm_head GEMVs read the INT8 rows with their scales."""
    from oracle import golden as G
    cfg = G.CFG_TINY
    base = G.make_base_weights(cfg, 81, round_fp16=True)
    lora = G.make_lora(cfg, 82)
    prompt = G.make_tokens(cfg, 1, 16, 83)[0][0]
    ctx = _ctx(llmcu, G, cfg, base, lora, max_seq=64, int8=True)
    _check(G, cfg, ctx, _int8_view(base), lora, prompt, 6)
    ctx.close()


def test_generate_rejects_overlong_requests(llmcu, cuda_device):
    from oracle import golden as G
    cfg = G.CFG_TINY
    ctx = _ctx(llmcu, G, cfg, G.make_base_weights(cfg, 1, round_fp16=True), G.make_lora(cfg, 2), max_seq=32)
    with pytest.raises(llmcu.LlmcuError):
        ctx.generate(np.arange(30, dtype=np.int32), 3)
    with pytest.raises(llmcu.LlmcuError):
        ctx.generate(np.array([5000], dtype=np.int32), 2)  # id outside the tiny vocabulary
    toks, _, _ = ctx.generate(np.arange(30, dtype=np.int32), 2)  # the context still works
    assert toks.shape == (2,)
    ctx.close()
