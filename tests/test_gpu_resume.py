"""Checkpoint / resume on the GPU: an AdamW-moment sidecar beside the
reference's adapter files (the reference saves A and B only and cannot
resume).

A run that saves adapters + AdamW moments after step 2 and is continued in a
fresh context from those files must take step 3 as the uninterrupted run
does.  The step's gradient sums are not bit-reproducible (fp32 atomics and
TMA reduce-adds in no fixed order, whose last-bit differences can flip an
fp16 rounding downstream), so two identical runs agree to about 1e-3 in the
gradients and AdamW moments.  In the adapters most elements agree to ~1e-4,
but an element whose gradient sits at the noise floor can take Adam's
~lr * sign(g) step in the other direction (2 lr apart: 1.9e-3 relative on a
tiny-shape B once in a handful of runs).  The checks therefore use 1e-2 (the
gradient parity bound) on adapters and on moments -- a resume that lost the
moments would miss the first two steps' share of m (tens of percent).  The
sidecar refuses a context of another shape, and the C++ driver's --resume
continues a synthetic run to the same adapters."""
import os
import subprocess

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
INVALID_ARG, IO = 1, 4


def _ctx(llmcu, G, cfg, batch, seq, seed, lora_seed=None):
    model = llmcu.Model(cfg.hidden, cfg.n_layers, cfg.n_heads, cfg.n_kv_heads, cfg.head_dim, cfg.ffn, cfg.vocab,
                        cfg.rope_theta, cfg.rms_eps)
    ctx = llmcu.Context(model, llmcu.Lora(cfg.lora_rank, cfg.lora_alpha), llmcu.Run(batch, seq))
    ctx.set_base(G.make_base_weights(cfg, seed, round_fp16=True))
    ctx.set_lora_dict(G.make_lora(cfg, seed + 1 if lora_seed is None else lora_seed))
    return ctx


def _close(a, b, rtol=1e-2):
    for k in a:
        d = np.linalg.norm(a[k] - b[k]) / max(np.linalg.norm(b[k]), 1e-30)
        assert d <= rtol, (k, d)


def test_resume_continues_the_run(llmcu, cuda_device, tmp_path):
    from oracle import golden as G
    cfg = G.CFG_TINY
    batch, seq, seed = 2, 48, 5
    toks = [G.make_tokens(cfg, batch, seq, seed + 10 + s) for s in range(3)]
    opt = llmcu.AdamW()
    a = _ctx(llmcu, G, cfg, batch, seq, seed)
    for step in (1, 2):
        a.train_step(toks[step - 1][0], toks[step - 1][1], opt, step)
    a.save_lora(str(tmp_path), 2)
    a.save_adamw_state(str(tmp_path), 2)
    assert os.path.getsize(tmp_path / "lora_step2_adamw.bin") == 64 + 2 * 4 * a.lora_param_count()
    a.train_step(toks[2][0], toks[2][1], opt, 3)
    want = a.lora_dict()

    def moments(ctx, name):  # (m, v) after step 3, through the sidecar writer
        d = tmp_path / name
        d.mkdir()
        ctx.save_adamw_state(str(d), 3)
        raw = np.fromfile(d / "lora_step3_adamw.bin", dtype=np.float32)[16:]
        return raw[: raw.size // 2], raw[raw.size // 2:]

    m_want, v_want = moments(a, "a")
    b = _ctx(llmcu, G, cfg, batch, seq, seed, lora_seed=seed + 100)  # other adapters before the load
    b.load_lora(str(tmp_path), 2)
    b.load_adamw_state(str(tmp_path), 2)
    b.train_step(toks[2][0], toks[2][1], opt, 3)
    _close(b.lora_dict(), want)
    m_b, v_b = moments(b, "b")
    assert G.rel_l2(m_b, m_want) <= 1e-2 and G.rel_l2(v_b, v_want) <= 1e-2

    # without the moments the step starts Adam afresh: m lacks the first two
    # steps' share (beta1 weights them 0.9 and 0.81)
    c = _ctx(llmcu, G, cfg, batch, seq, seed)
    c.load_lora(str(tmp_path), 2)
    c.train_step(toks[2][0], toks[2][1], opt, 3)
    m_c, _ = moments(c, "c")
    assert G.rel_l2(m_c, m_want) > 0.1


def test_sidecar_refuses_other_shapes(llmcu, cuda_device, tmp_path):
    from oracle import golden as G
    cfg = G.CFG_TINY
    a = _ctx(llmcu, G, cfg, 1, 32, 3)
    a.save_adamw_state(str(tmp_path), 7)
    lib = llmcu.lib()
    # wrong step number in the file name -> missing file
    assert lib.llmcu_load_adamw_state(a._h, str(tmp_path).encode(), 8) == IO
    # another rank
    model = llmcu.Model(cfg.hidden, cfg.n_layers, cfg.n_heads, cfg.n_kv_heads, cfg.head_dim, cfg.ffn, cfg.vocab,
                        cfg.rope_theta, cfg.rms_eps)
    other = llmcu.Context(model, llmcu.Lora(cfg.lora_rank * 2, cfg.lora_alpha), llmcu.Run(1, 32))
    assert lib.llmcu_load_adamw_state(other._h, str(tmp_path).encode(), 7) == INVALID_ARG
    assert b"rank" in lib.llmcu_last_error(other._h)
    # a truncated file
    path = tmp_path / "lora_step7_adamw.bin"
    data = path.read_bytes()
    path.write_bytes(data[: len(data) // 2])
    assert lib.llmcu_load_adamw_state(a._h, str(tmp_path).encode(), 7) == IO


def test_driver_resume_matches_uninterrupted_run(cuda_device, tmp_path):
    exe = os.path.join(ROOT, "llm.cu_b200", "llm_train")
    if not os.path.exists(exe):
        pytest.skip("llm_train not built")
    common = ["--config", "tiny", "--synthetic", "--seq-len", "32", "--batch", "2", "--log-every", "1", "--seed", "9"]
    full, part = tmp_path / "full", tmp_path / "part"
    full.mkdir()
    part.mkdir()
    env = dict(os.environ, WORLD_SIZE="1", RANK="0", LOCAL_RANK="0")
    subprocess.run([exe, *common, "--steps", "4", "--save-every", "4", "--out", str(full)], check=True, env=env,
                   timeout=300)
    subprocess.run([exe, *common, "--steps", "2", "--save-every", "2", "--out", str(part)], check=True, env=env,
                   timeout=300)
    out = subprocess.run([exe, *common, "--steps", "4", "--save-every", "4", "--resume", "2", "--out", str(part)],
                         check=True, env=env, timeout=300, capture_output=True, text=True).stdout
    assert "Resumed from step 2" in out
    assert "step    3" in out and "step    1" not in out
    names = sorted(f for f in os.listdir(full) if f.startswith("lora_step4_") and f.endswith(".bin"))
    assert len(names) == 2 * 4 * 2 + 1  # tiny: 2 layers x 4 projections x (A, B) + the AdamW sidecar
    for f in names:
        x = np.fromfile(full / f, dtype=np.float32)
        y = np.fromfile(part / f, dtype=np.float32)
        tol = 1e-2
        if f.endswith("_adamw.bin"):
            x, y = x[16:], y[16:]  # past the 64-byte header
            tol = 1e-2
        assert x.shape == y.shape
        assert np.linalg.norm(x - y) <= tol * max(np.linalg.norm(x), 1e-30), f
