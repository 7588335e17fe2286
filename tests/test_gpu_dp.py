"""Data parallelism through the C ABI: one process per GPU, LoRA gradients
summed over the ranks by the library's NCCL all-reduce, identical AdamW on
every rank.  The ranks together must reproduce the fp32 golden of the whole
batch (loss 1e-3 relative; gradients and post-AdamW adapters rel-L2 <= 1e-2,
cosine >= 0.999) and agree with one another bit for bit.

The failure test makes the failure on the host: a group whose second rank
never joins must end with an error status from the init deadline, not hang."""
import os
import subprocess
import sys

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _n_gpus():
    import torch
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


@pytest.mark.parametrize("world,projs", [(2, ("wq", "wk", "wv", "wo")),
                                         (2, ("wq", "wk", "wv", "wo", "w_gate", "w_up", "w_down")),
                                         (4, ("wq", "wk", "wv", "wo")),
                                         (8, ("wq", "wk", "wv", "wo"))])
def test_dp_ranks_match_golden(llmcu, cuda_device, tmp_path, world, projs):
    if _n_gpus() < world:
        pytest.skip(f"needs {world} GPUs")
    from oracle import golden as G
    batch, seq, seed = 2, 48, 31
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    idfile = str(tmp_path / "nccl.id")
    procs = [subprocess.Popen([sys.executable, os.path.join(ROOT, "tests", "dp_rank.py"), "--rank", str(r),
                               "--world", str(world), "--idfile", idfile, "--out", str(tmp_path / f"r{r}.npz"),
                               "--batch", str(batch), "--seq", str(seq), "--seed", str(seed),
                               "--targets", ",".join(projs)], env=env)
             for r in range(world)]
    for p in procs:
        assert p.wait(timeout=600) == 0
    outs = [dict(np.load(tmp_path / f"r{r}.npz")) for r in range(world)]

    cfg = G.CFG_TINY
    base = G.make_base_weights(cfg, seed, round_fp16=True)
    lora = G.make_lora(cfg, seed + 1, projs=projs)
    tok, tgt = G.make_tokens(cfg, batch * world, seq, seed + 2)
    ref = G.forward_backward(cfg, base, lora, tok, tgt)
    upd = {k: a.copy() for k, a in lora.items()}
    opt = llmcu.AdamW()
    G.adamw(upd, ref.grads, G.zeros_like_lora(lora), G.zeros_like_lora(lora), lr=opt.lr, beta1=opt.beta1,
            beta2=opt.beta2, eps=opt.eps, wd=opt.weight_decay, step=1)
    for o in outs:
        assert abs(float(o["loss"]) - ref.loss) <= 1e-3 * abs(ref.loss)
        for k in ref.grads:
            g = o["g_" + k]
            assert G.rel_l2(g, ref.grads[k]) <= 1e-2 and G.cosine(g, ref.grads[k]) >= 0.999, k
            p = o["p_" + k]
            assert G.rel_l2(p, upd[k]) <= 1e-2 and G.cosine(p, upd[k]) >= 0.999, k
    for o in outs[1:]:
        for k in outs[0]:
            assert np.array_equal(outs[0][k], o[k]), k


def test_dp_missing_rank_fails_by_deadline(llmcu, cuda_device):
    """World of 2 with only rank 0 present: dp_init gives up after its timeout."""
    import time
    cfg = llmcu.Model.tiny()
    ctx = llmcu.Context(cfg, llmcu.Lora(4, 8.0), llmcu.Run(1, 32))
    uid = llmcu.Context.dp_unique_id()
    ctx.dp_set_timeout_ms(3000)
    t0 = time.time()
    with pytest.raises(llmcu.LlmcuError) as ei:
        ctx.dp_init(uid, 0, 2)
    assert time.time() - t0 < 60
    inv = {v: k for k, v in llmcu.STATUS.items()}
    assert ei.value.status in (inv["NCCL"], inv["TIMEOUT"])
    # the context stays usable as a single-GPU trainer
    tok = np.zeros((1, 32), np.int32)
    loss = ctx.forward_backward(tok, tok)
    assert np.isfinite(loss)
    ctx.close()
