"""One CPU rank of the data-parallel host-logic test (tests/test_dp_gloo.py
starts WORLD_SIZE of these over gloo on 127.0.0.1; no GPU, no NCCL).

Checks, on every rank:
* bench.py's rank plumbing -- the max-over-ranks timing reduction, the NCCL
  unique-id hand-out (only rank 0 creates it) and the per-rank token shards
  (seed 1000 + r: distinct across ranks, reproducible per rank);
* the decomposition the library's NCCL path relies on: each rank scales its
  local NLL sum by 1 / (positions over all ranks) and the ranks' LoRA
  gradients are summed (llmcu_dp_init + the per-layer ncclAllReduce in
  run_forward_backward).  With the CPU oracle as each rank's step, the summed
  shard gradients and the summed shard losses must equal the oracle's
  full-batch gradients and loss, and AdamW on the summed gradients must leave
  every rank with bit-identical adapters.
Any failed check raises, so the process exits non-zero."""
import datetime
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def main():
    import torch
    import torch.distributed as dist

    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.set_num_threads(2)
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=60))
    import bench
    from oracle import golden as G

    # --- timing: every rank reports the slowest rank's figure
    got = bench.rank_max(dist, world, 1.5 * (rank + 1))
    assert got == 1.5 * world, got

    # --- unique id: rank 0 makes it, everyone receives the same bytes
    def make_id():
        assert rank == 0, "only rank 0 may create the NCCL id"
        return bytes(range(128))
    uid = bench.share_unique_id(dist, rank, world, make_id)
    assert uid == bytes(range(128))

    # --- token shards: one full batch per rank, distinct, reproducible
    vocab, B, S = 151936, 8, 64
    tok, tgt = bench.make_tokens(vocab, B, S, bench.shard_seed(rank), "zipf")
    tok2, _ = bench.make_tokens(vocab, B, S, bench.shard_seed(rank), "zipf")
    assert np.array_equal(tok, tok2)
    assert np.array_equal(tok[:, 1:], tgt[:, :-1])
    shards = [None] * world
    dist.all_gather_object(shards, tok)
    for r in range(world):
        if r != rank:
            assert not np.array_equal(shards[r], tok), (rank, r)

    # --- gradient decomposition over the CPU oracle
    cfg = G.CFG_TINY
    b, seq = 2, 32
    projs = G.ALL_PROJS
    base = G.make_base_weights(cfg, 91, round_fp16=True)
    lora = G.make_lora(cfg, 92, projs=projs, b_std=0.05)
    ftok, ftgt = G.make_tokens(cfg, b * world, seq, 93, dist="zipf")
    rows = slice(rank * b, (rank + 1) * b)
    local = G.forward_backward(cfg, base, lora, ftok[rows], ftgt[rows])
    n_total = local.n_positions * world          # equal shards: (S - 1) positions per sequence
    scale = local.n_positions / n_total          # local mean -> local share of the global mean
    keys = sorted(local.grads)
    flat = torch.from_numpy(np.concatenate([local.grads[k].ravel() for k in keys]) * np.float32(scale))
    dist.all_reduce(flat, op=dist.ReduceOp.SUM)
    loss = torch.tensor([local.loss * scale], dtype=torch.float64)
    dist.all_reduce(loss, op=dist.ReduceOp.SUM)
    summed, off = {}, 0
    for k in keys:
        n = local.grads[k].size
        summed[k] = flat[off:off + n].numpy().reshape(local.grads[k].shape)
        off += n

    full = G.forward_backward(cfg, base, lora, ftok, ftgt)
    assert abs(float(loss.item()) - full.loss) <= 1e-6 * abs(full.loss), (float(loss.item()), full.loss)
    assert set(summed) == set(full.grads)
    for k in keys:
        r = G.rel_l2(summed[k], full.grads[k])
        assert r <= 1e-5, f"rank {rank} {k}: rel_l2 {r:.3e}"

    upd = {k: a.copy() for k, a in lora.items()}
    G.adamw(upd, summed, G.zeros_like_lora(lora), G.zeros_like_lora(lora), lr=3e-4, beta1=0.9, beta2=0.999,
            eps=1e-8, wd=0.01, step=1)
    mine = np.concatenate([upd[k].ravel() for k in keys])
    every = [None] * world
    dist.all_gather_object(every, mine)
    for r in range(world):
        assert np.array_equal(every[r], mine), f"adapters of rank {r} differ from rank {rank}'s"
    ref = {k: a.copy() for k, a in lora.items()}
    G.adamw(ref, full.grads, G.zeros_like_lora(lora), G.zeros_like_lora(lora), lr=3e-4, beta1=0.9,
            beta2=0.999, eps=1e-8, wd=0.01, step=1)
    for k in keys:
        r = G.rel_l2(upd[k], ref[k])
        assert r <= 1e-2, f"post-adamw {k}: rel_l2 {r:.3e}"

    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
