"""One rank of the data-parallel parity test (tests/test_gpu_dp.py starts one
process per GPU).  Rank r takes sequences [r*b, (r+1)*b) of a seeded batch,
joins the NCCL group through the library's own entry points (the unique id
travels through a file), runs one forward+backward and one AdamW step, and
saves its loss, LoRA gradients and updated adapters."""
import argparse
import os
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "tests"))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--rank", type=int, required=True)
    ap.add_argument("--world", type=int, required=True)
    ap.add_argument("--idfile", required=True)
    ap.add_argument("--out", required=True)
    ap.add_argument("--batch", type=int, default=2, help="sequences per rank")
    ap.add_argument("--seq", type=int, default=48)
    ap.add_argument("--seed", type=int, default=31)
    ap.add_argument("--targets", default="wq,wk,wv,wo", help="adapted projections (comma list)")
    a = ap.parse_args()
    projs = tuple(a.targets.split(","))

    from conftest import load_binding
    from oracle import golden as G
    llmcu = load_binding()
    cfg = G.CFG_TINY
    base = G.make_base_weights(cfg, a.seed, round_fp16=True)
    lora = G.make_lora(cfg, a.seed + 1, projs=projs)
    tok, tgt = G.make_tokens(cfg, a.batch * a.world, a.seq, a.seed + 2)
    rows = slice(a.rank * a.batch, (a.rank + 1) * a.batch)
    model = llmcu.Model(cfg.hidden, cfg.n_layers, cfg.n_heads, cfg.n_kv_heads, cfg.head_dim, cfg.ffn, cfg.vocab,
                        cfg.rope_theta, cfg.rms_eps)
    ctx = llmcu.Context(model, llmcu.Lora(cfg.lora_rank, cfg.lora_alpha, llmcu.targets_mask(projs)),
                        llmcu.Run(a.batch, a.seq), device=a.rank)
    ctx.set_base(base)
    ctx.set_lora_dict(lora)
    if a.rank == 0:
        tmp = a.idfile + ".tmp"
        with open(tmp, "wb") as f:
            f.write(llmcu.Context.dp_unique_id())
        os.replace(tmp, a.idfile)
    t0 = time.time()
    while not os.path.exists(a.idfile):
        if time.time() - t0 > 60:
            raise SystemExit("no NCCL id from rank 0")
        time.sleep(0.05)
    with open(a.idfile, "rb") as f:
        uid = f.read()
    ctx.dp_set_timeout_ms(60000)
    ctx.dp_init(uid, a.rank, a.world)
    loss = ctx.forward_backward(tok[rows], tgt[rows])
    grads = ctx.grads_dict()
    ctx.adamw(llmcu.AdamW(), step=1)
    after = ctx.lora_dict()
    np.savez(a.out, loss=np.float64(loss), **{"g_" + k: v for k, v in grads.items()},
             **{"p_" + k: v for k, v in after.items()})
    ctx.close()


if __name__ == "__main__":
    main()
