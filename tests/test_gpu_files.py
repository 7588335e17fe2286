"""The reference's file interfaces on the GPU path.

* Adapter files: llmcu_save_lora (device adapters -> files) writes exactly the
  bytes of the host-side writer that tests/test_lora_files.py runs the
  reference's unmodified python/save_lora.py against, at the Qwen3-1.7B
  dimensions save_lora.py hard-codes; llmcu_load_lora reads such files back
  into the context (src/train.cu:146-170, python/save_lora.py:47-57,81-113).
* Training data and base weights: the llm_train driver, given a
  data/train_tokens.bin (int32 count + ids, python/tokenize_input.py:22-26)
  and a directory of fp32 weight files named as src/train.cu:56-89 loads
  them, takes the reference's windows (src/train.cu:195-214,251-258) and its
  logged losses match the golden's on the same windows, weights and
  adapters."""
import os
import re
import subprocess

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LOSS_RTOL = 1e-3


def test_save_lora_writes_the_host_writer_bytes_at_1p7b_dims(llmcu, cuda_device, tmp_path):
    from oracle import golden as G
    cfg = G.CFG_QWEN3_1P7B
    model = llmcu.Model.qwen3_1p7b()
    lora_cfg = llmcu.Lora(cfg.lora_rank, cfg.lora_alpha)
    lora = G.make_lora(cfg, 61)
    ctx = llmcu.Context(model, lora_cfg, llmcu.Run(1, 16))
    try:
        ctx.set_lora_dict(lora)
        a, b = tmp_path / "device", tmp_path / "host"
        a.mkdir()
        b.mkdir()
        ctx.save_lora(str(a), 100)
        llmcu.LoraFiles(model, lora_cfg).write(lora, str(b), 100)
        names = sorted(os.listdir(a))
        assert names == sorted(os.listdir(b)) and len(names) == cfg.n_layers * 4 * 2
        for n in names:
            assert (a / n).read_bytes() == (b / n).read_bytes(), n
        # files from elsewhere (as save_lora.py --from-hf writes them) load into the context
        other = G.make_lora(cfg, 62)
        llmcu.LoraFiles(model, lora_cfg).write(other, str(b), 7)
        ctx.load_lora(str(b), 7)
        got = ctx.lora_dict()
        assert all(np.array_equal(got[k], other[k]) for k in other)
    finally:
        ctx.close()


def _write_weight_dir(base, cfg, d):
    """fp32 weight files with the names src/train.cu:56-89 reads."""
    names = {"attn_norm": "input_layernorm.weight", "ffn_norm": "post_attention_layernorm.weight",
             "wq": "self_attn.q_proj.weight", "wk": "self_attn.k_proj.weight", "wv": "self_attn.v_proj.weight",
             "wo": "self_attn.o_proj.weight", "q_norm": "self_attn.q_norm.weight", "k_norm": "self_attn.k_norm.weight",
             "w_gate": "mlp.gate_proj.weight", "w_up": "mlp.up_proj.weight", "w_down": "mlp.down_proj.weight"}
    base["embed"].astype(np.float32).tofile(d / "model.embed_tokens.weight.bin")
    base["final_norm"].astype(np.float32).tofile(d / "model.norm.weight.bin")
    for l in range(cfg.n_layers):
        for k, n in names.items():
            base[f"L{l}.{k}"].astype(np.float32).tofile(d / f"model.layers.{l}.{n}.bin")


def test_llm_train_on_data_and_weight_files_matches_golden(llmcu, cuda_device, tmp_path):
    exe = os.path.join(ROOT, "llm.cu_b200", "llm_train")
    if not os.path.exists(exe):
        pytest.skip("llm_train not built")
    from oracle import golden as G
    cfg = G.CFG_TINY
    rng = np.random.Generator(np.random.PCG64(71))
    base = G.make_base_weights(cfg, 72, round_fp16=True)
    # non-unit norm gains, so that a gain file read into the wrong slot shows
    for k in base:
        if base[k].ndim == 1:
            base[k] = (1.0 + 0.1 * rng.standard_normal(base[k].shape)).astype(np.float32)
    wdir = tmp_path / "weights"
    wdir.mkdir()
    _write_weight_dir(base, cfg, wdir)
    S, B, steps = 32, 2, 2
    ids = rng.integers(0, cfg.vocab, size=5 * (S + 1) + 3, dtype=np.int64).astype(np.int32)
    data = tmp_path / "train_tokens.bin"
    with open(data, "wb") as f:
        np.array([ids.size], np.int32).tofile(f)
        ids.tofile(f)
    seed = 9
    out = tmp_path / "out"
    out.mkdir()
    env = dict(os.environ, WORLD_SIZE="1", RANK="0", LOCAL_RANK="0")
    log = subprocess.run([exe, "--config", "tiny", "--weights", str(wdir), "--data", str(data), "--seq-len", str(S),
                          "--batch", str(B), "--steps", str(steps), "--log-every", "1", "--seed", str(seed), "--out",
                          str(out)], check=True, env=env, timeout=300, capture_output=True, text=True).stdout
    assert f"Loaded {ids.size} training tokens" in log
    losses = [float(x) for x in re.findall(r"step\s+\d+\s+loss\s+([0-9.]+)", log)]
    assert len(losses) == steps
    # the driver's adapters: llmcu_init_lora_synthetic(seed + 1, 0.01) on the device
    model = llmcu.Model(cfg.hidden, cfg.n_layers, cfg.n_heads, cfg.n_kv_heads, cfg.head_dim, cfg.ffn, cfg.vocab,
                        cfg.rope_theta, cfg.rms_eps)
    with llmcu.Context(model, llmcu.Lora(cfg.lora_rank, cfg.lora_alpha), llmcu.Run(1, S)) as ctx:
        ctx.init_lora_synthetic(seed=seed + 1, b_std=0.01)
        lora = ctx.lora_dict()
    m, v = G.zeros_like_lora(lora), G.zeros_like_lora(lora)
    n_seqs = ids.size // (S + 1)
    opt = llmcu.AdamW()
    for step in range(1, steps + 1):
        win = [((step - 1) * B + b) % n_seqs for b in range(B)]  # src/train.cu:251-258, B per step
        tok = np.stack([ids[w * (S + 1): w * (S + 1) + S] for w in win])
        tgt = np.stack([ids[w * (S + 1) + 1: w * (S + 1) + S + 1] for w in win])
        r = G.train_step(cfg, base, lora, m, v, tok, tgt, lr=opt.lr, step=step)
        assert abs(losses[step - 1] - r.loss) <= LOSS_RTOL * abs(r.loss) + 1e-4, (step, losses, r.loss)
    # the saved adapters after the last step follow the golden's
    got = llmcu.LoraFiles(model, llmcu.Lora(cfg.lora_rank, cfg.lora_alpha)).read(str(out), steps)
    for k in lora:
        assert G.rel_l2(got[k], lora[k]) <= 1e-2, k
