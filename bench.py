#!/usr/bin/env python
"""bench.py -- LoRA training-step throughput of the B200 build (libllmcu.so).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload c2|c1|c3|c4]
                    [--lora-targets attn|mlp|all|wq,...,w_down] [--int8-in-gemm] [--decode N [--int8]]

One step = forward + cross-entropy + backward + AdamW of the Qwen3-1.7B-shape
LoRA model on one batch of synthetic tokens per GPU.
Default workload c2: batch 8 per GPU x seq 512, Zipf(1.1) token ids, fp16 base
~N(0, 0.02) drawn on the device, LoRA rank 16 / alpha 32 adapters.  For N > 1
(torchrun, one process per GPU) the batch is sharded (8 sequences per rank,
rank r draws with seed + r) and the LoRA gradients are allreduced over NCCL
inside the library; `value` is the whole-job tokens/s with the time taken as
the max over ranks.

Printed JSON line keys beyond the driver contract:
  e2e        the same metric through the public host-buffer API
             (llmcu_train_step: H2D of tokens/targets + D2H of the loss each step)
  roofline   tcgen05 GEMM class: algorithmic GEMM FLOPs per launch / measured
             time per launch (CUDA events on the library's compute stream)
  cpu_baseline  the fp32 CPU autograd golden (oracle/golden.py) on a bounded
             sample, rank 0 at N = 1 only
  kernels    per-class device time per step from the same event pass
  clocks     nvidia-smi samples taken during the timed region

--lora-targets trains adapters on other projections than the reference's
q/k/v/o (the MLP's too with `all`); --int8-in-gemm (c4) lets the GEMMs stage
the INT8 codes instead of one dequantisation pass per weight; --decode N times
greedy KV-cache generation of N tokens after a 128-token prompt instead of the
training step.
"""
from __future__ import annotations

import argparse
import importlib.util
import json
import os
import shutil
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "LoRA fine-tune tokens/s per box, Qwen3-1.7B shape"
UNIT = "tokens/s"
WORKLOADS = {
    # name: (batch per GPU, seq, token dist, base dtype, description)
    "c2": (8, 512, "zipf", 0, "qwen3-1.7b-shape LoRA r16 step, batch 8/GPU x seq 512, Zipf(1.1) tokens, fp16 base"),
    "c1": (1, 128, "zipf", 0, "qwen3-1.7b-shape LoRA r16 step, batch 1 x seq 128, Zipf(1.1) tokens, fp16 base"),
    "c3": (1, 4096, "uniform", 0, "qwen3-1.7b-shape LoRA r16 step, batch 1/GPU x seq 4096, uniform tokens, fp16 base"),
    "c4": (8, 512, "zipf", 1, "qwen3-1.7b-shape LoRA r16 step, batch 8/GPU x seq 512, Zipf(1.1) tokens, INT8 base"),
}


def load_binding():
    spec = importlib.util.spec_from_file_location("llmcu", os.path.join(ROOT, "llm.cu_b200", "llmcu.py"))
    mod = importlib.util.module_from_spec(spec)
    sys.modules["llmcu"] = mod
    spec.loader.exec_module(mod)
    return mod


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained", d["bf16_tflops"]), "src": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "src": "fallback"}


class ClockSampler:
    """nvidia-smi clocks/throttle samples during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.proc = None
        self.path = None
        if shutil.which("nvidia-smi") is None:
            return
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        self.proc = subprocess.Popen(["nvidia-smi", "-i", str(gpu_index), f"--query-gpu={self.FIELDS}",
                                      "--format=csv,noheader,nounits", "-lms", "200"],
                                     stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)

    def stop(self):
        if self.proc is None:
            return None
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        with open(self.path) as f:
            lines = f.readlines()
        os.unlink(self.path)
        return self.summarise(lines)

    @staticmethod
    def summarise(lines):
        """Median SM clock, max clock, the throttle reasons seen active and
        the peak power of `--format=csv,noheader,nounits` rows of FIELDS."""
        rows = []
        for line in lines:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) >= 9:
                rows.append(parts)
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": float(rows[0][2]) if rows[0][2].replace(".", "").isdigit() else None,
                "reasons": reasons, "samples": len(rows),
                "power_w_max": max((float(r[3]) for r in rows if r[3].replace(".", "").isdigit()), default=None)}


def layer_gemm_flops_per_token(m) -> float:
    """Forward + dX of the frozen linears of every layer (the gemm_tc class)."""
    H, Q, KV, I, L = m.hidden, m.n_heads * m.head_dim, m.n_kv_heads * m.head_dim, m.ffn, m.n_layers
    return float(4 * L * (Q * H + 2 * KV * H + H * Q + 3 * I * H))


def lm_head_flops_per_token(m) -> float:
    """Forward + dX of the tied lm_head (the lm_head class: logits and d_xf)."""
    return float(4 * m.vocab * m.hidden)


def algorithmic_gemm_flops_per_token(m) -> float:
    """Forward + dX of every frozen linear (tied lm_head once)."""
    return layer_gemm_flops_per_token(m) + lm_head_flops_per_token(m)


def algorithmic_flops_per_token(m, seq, n_lora) -> float:
    """The step's algorithmic work per token: 4 N_lin (forward + dX of the
    frozen linears) + 3 (2 S hd nq L) (causal attention forward and backward)
    + 6 n_lora (adapter forward, dX and gradients)."""
    attn = 3 * (2 * seq * m.head_dim * m.n_heads * m.n_layers)
    return algorithmic_gemm_flops_per_token(m) + attn + 6.0 * n_lora


ALL_PROJS = ("wq", "wk", "wv", "wo", "w_gate", "w_up", "w_down")


def parse_targets(arg: str):
    """Adapter names of a --lora-targets value."""
    named = {"attn": ALL_PROJS[:4], "mlp": ALL_PROJS[4:], "all": ALL_PROJS}
    if arg in named:
        return tuple(named[arg])
    out = tuple(x.strip() for x in arg.split(",") if x.strip())
    bad = [x for x in out if x not in ALL_PROJS]
    if bad or not out:
        raise SystemExit(f"unknown --lora-targets entries: {bad or arg}")
    return tuple(p for p in ALL_PROJS if p in out)


def make_tokens(vocab, batch, seq, seed, dist):
    rng = np.random.Generator(np.random.PCG64(seed))
    n = batch * (seq + 1)
    if dist == "uniform":
        ids = rng.integers(0, vocab, size=n, dtype=np.int64)
    else:
        k = np.arange(1, vocab + 1, dtype=np.float64)
        cdf = np.cumsum(k ** -1.1)
        cdf /= cdf[-1]
        ids = np.minimum(np.searchsorted(cdf, rng.random(n), side="right"), vocab - 1)
    win = ids.reshape(batch, seq + 1).astype(np.int32)
    return np.ascontiguousarray(win[:, :seq]), np.ascontiguousarray(win[:, 1:])


def shard_seed(rank: int) -> int:
    """Rank r of a data-parallel run draws its own sequences with seed 1000 + r
    (weak scaling: every rank adds one full batch of distinct tokens)."""
    return 1000 + rank


def rank_max(dist_, world: int, x: float) -> float:
    """Max of a per-rank float over the host process group (gloo): the timed
    figure of an N-GPU run is the slowest rank's."""
    if world == 1:
        return x
    import torch
    t = torch.tensor([x], dtype=torch.float64)
    dist_.all_reduce(t, op=dist_.ReduceOp.MAX)
    return float(t.item())


def share_unique_id(dist_, rank: int, world: int, make_id) -> bytes:
    """Rank 0 creates the NCCL unique id (make_id, the library's
    llmcu_dp_get_unique_id) and every rank receives it over the host process
    group; the other ranks never call make_id."""
    if world == 1:
        return make_id()
    obj = [make_id() if rank == 0 else None]
    dist_.broadcast_object_list(obj, src=0)
    return obj[0]


def cpu_baseline(seq):
    """fp32 CPU autograd golden on a bounded sample: 2 layers of the full
    shape (full vocabulary), batch 1 x seq, one warm-up + timed steps; the
    tokens/s is scaled to the 28-layer model by the FLOP ratio."""
    import torch
    from oracle import golden as G
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    full = G.CFG_QWEN3_1P7B
    cfg = G.layer_slice(full, 2)
    base = G.make_base_weights(cfg, 7, round_fp16=True)
    lora = G.make_lora(cfg, 8)
    tok, tgt = G.make_tokens(cfg, 1, seq, 9, dist="zipf")
    G.forward_backward(cfg, base, lora, tok, tgt)
    times = []
    t_budget = time.time() + 20.0
    while len(times) < 3 and (not times or time.time() < t_budget):
        t0 = time.perf_counter()
        G.forward_backward(cfg, base, lora, tok, tgt)
        times.append(time.perf_counter() - t0)
    t = statistics.median(times)
    sample_tps = seq / t
    ratio = G.algorithmic_flops_per_token(cfg, seq) / G.algorithmic_flops_per_token(full, seq)
    return {"value": round(sample_tps * ratio, 3), "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"oracle/golden.py fp32 torch-CPU autograd, 2 of 28 layers at full shape (vocab 151936), "
                      f"batch 1 x seq {seq}, median of {len(times)} steps ({t:.2f} s), scaled to 28 layers by "
                      f"the algorithmic-FLOP ratio {ratio:.4f}",
            "sample_tokens_per_s": round(sample_tps, 3)}


def run_reference(args, workload):
    """The reference trainer's own CUDA code (compiled from its sources into
    oracle/_ref by oracle/ref_harness/Makefile) on one GPU, rank 0 only: the
    whole batch of the workload per step (the reference runs its B sequences
    one after another, src/train.cu:251-291 per sequence, then one AdamW), on
    the same token windows as this arm's rank 0 (make_tokens, seed
    shard_seed(0))."""
    B, S, dist, base_dtype, desc = WORKLOADS[workload]
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    exe = os.path.join(ROOT, "oracle", "_ref", "ref_harness_full")
    line = {"metric": METRIC, "unit": UNIT, "higher_is_better": True, "impl": "reference", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "config": {"workload": workload, "description": desc, "global_batch": B,
                                            "seq_len": S}}
    if not os.path.exists(exe):
        line["unavailable"] = "oracle/_ref/ref_harness_full was not built (make -C oracle/ref_harness)"
        print(json.dumps(line))
        return 0
    vocab = 151936
    tok, tgt = make_tokens(vocab, B, S, shard_seed(0), dist)
    windows = np.concatenate([tok, tgt[:, -1:]], axis=1).astype(np.int32)  # [B, S + 1]
    fd, tok_path = tempfile.mkstemp(suffix=".i32")
    os.close(fd)
    windows.tofile(tok_path)
    try:
        cmd = [exe, "bench", str(B), str(S), str(args.steps), str(args.warmup), tok_path]
        t0 = time.perf_counter()
        r = subprocess.run(cmd, capture_output=True, text=True, timeout=3000)
        wall = time.perf_counter() - t0
    finally:
        os.unlink(tok_path)
    if r.returncode != 0:
        line["unavailable"] = f"reference harness exited {r.returncode}: {r.stderr.strip()[-200:]}"
        print(json.dumps(line))
        return 0
    res = json.loads(r.stdout.strip().splitlines()[-1])
    v = res["tokens_per_s"]
    line.update({"value": round(v, 3), "ms_per_step": round(res["ms_per_step"], 3), "loss": res.get("loss"),
                 "wall_s": round(wall, 1),
                 "e2e": {"value": round(v, 3), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
                 "cpu_baseline": {"value": round(v, 3), "unit": UNIT, "cores": 1, "kind": "reference",
                                  "sample": f"reference trainer's own CUDA code (visheshnarayan/llm.cu src/kernels/"
                                            f"*.cu, compute_80 PTX JIT on the B200) via oracle/_ref/ref_harness_full,"
                                            f" the whole batch of {B} x seq {S} per step (its sequences one after "
                                            f"another, then one AdamW), {dist} token windows identical to this "
                                            f"workload's rank 0, fp32, cudaEvent timing over {args.steps} steps"},
                 "gpu_launches": None})
    print(json.dumps(line))
    return 0


def run_decode(args):
    """`--decode N`: greedy KV-cache decoding of N tokens after a 128-token
    prompt on one GPU (llmcu_generate: batched prefill, then one CUDA-graph
    replay per token), Qwen3-1.7B shape, synthetic fp16 (or --int8) base.  Its
    own JSON line; not the training benchmark."""
    import torch
    torch.cuda.set_device(0)
    m = load_binding()
    model = m.Model.qwen3_1p7b(n_layers=args.layers)
    n_prompt, n_new = 128, args.decode
    base = m.BASE_INT8 if args.int8 else m.BASE_FP16
    ctx = m.Context(model, m.Lora(16, 32.0), m.Run(1, n_prompt + n_new, base), device=0)
    ctx.init_base_synthetic(seed=1, std=0.02)
    ctx.init_lora_synthetic(seed=2, b_std=0.01)
    prompt, _ = make_tokens(model.vocab, 1, n_prompt, 7, "zipf")
    ctx.generate(prompt[0], 8)  # warm-up: captures the decode graph
    runs = []
    for _ in range(max(1, args.steps)):
        _, _, ms = ctx.generate(prompt[0], n_new)
        runs.append(ms)
    ms = float(np.median(runs))
    # bytes every decoded token must read: all linear weights once (merged
    # q/k/v/o in fp16; MLP and lm_head fp16 or INT8 rows + scales) and the cache
    H, Q, KV, I, V, L = model.hidden, model.n_heads * model.head_dim, model.n_kv_heads * model.head_dim, \
        model.ffn, model.vocab, model.n_layers
    attn = (Q + 2 * KV) * H + H * Q
    mlp_el = 3 * I * H
    wbytes = L * (2 * attn + mlp_el * (1 if args.int8 else 2)) + V * H * (1 if args.int8 else 2)
    if args.int8:
        wbytes += L * (2 * I + H) * 4 + V * 4  # row scales
    avg_ctx = n_prompt + n_new / 2
    kv_bytes = L * 2 * avg_ctx * KV * 2
    bpt = wbytes + kv_bytes
    pk = peaks()
    achieved = bpt / (ms / 1e3) / 1e9
    line = {"metric": "greedy decode tokens/s, batch 1, Qwen3-1.7B shape", "value": round(1e3 / ms, 2),
            "unit": "tokens/s", "n_gpus": 1, "ms_per_token": round(ms, 4), "higher_is_better": True,
            "dtype": "int8 MLP/lm_head rows, fp16 q/k/v/o" if args.int8 else "f16",
            "data": "synthetic (device-generated base, seeded Zipf prompt)",
            "config": {"workload": "decode", "prompt": n_prompt, "new_tokens": n_new, "layers": L,
                       "base": "int8" if args.int8 else "fp16"},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": pk["hbm_gbs"], "unit": "GB/s",
                         "frac": round(achieved / pk["hbm_gbs"], 4), "bytes_per_token": int(bpt),
                         "peak_src": pk.get("src", "MEASURED_PEAKS.json")},
            "published_reference": "llm_engine 26.4 tok/s fp16, 33.8 tok/s int8 (RTX A5000, its README)"}
    print(json.dumps(line))
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="c2")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--layers", type=int, default=28,
                    help="fewer layers for small ncu captures only; the benchmark line uses 28")
    ap.add_argument("--decode", type=int, default=0,
                    help="instead of the training step: greedy decode of N tokens after a 128-token prompt")
    ap.add_argument("--int8", action="store_true", help="with --decode: INT8 base")
    ap.add_argument("--int8-in-gemm", action="store_true",
                    help="INT8 base (c4): the GEMMs stage the INT8 codes themselves instead of one dequant pass per weight")
    ap.add_argument("--deterministic", action="store_true",
                    help="fixed-order sums everywhere (per-key-tile dQ slabs): bit-identical repeated steps")
    ap.add_argument("--lm-head-chunk", type=int, default=0,
                    help="vocabulary columns per lm_head chunk (multiple of 256); 0 = the library's choice")
    ap.add_argument("--lora-targets", default="attn",
                    help="adapted projections: attn (the reference's q/k/v/o), mlp, all, or a comma list of "
                         "wq,wk,wv,wo,w_gate,w_up,w_down")
    args = ap.parse_args()
    if args.decode:
        return run_decode(args)
    if args.impl == "reference":
        return run_reference(args, args.workload)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        print(f"warning: --gpus {args.gpus} but WORLD_SIZE {world}; using WORLD_SIZE", file=sys.stderr)
    B, S, dist, base_dtype, desc = WORKLOADS[args.workload]

    import torch
    import torch.distributed as dist_
    torch.cuda.set_device(local)
    if world > 1:
        dist_.init_process_group("gloo", timeout=__import__("datetime").timedelta(seconds=300))

    def barrier():
        if world > 1:
            dist_.barrier()

    def max_over_ranks(x: float) -> float:
        return rank_max(dist_, world, x)

    m = load_binding()
    model = m.Model.qwen3_1p7b(n_layers=args.layers)
    projs = parse_targets(args.lora_targets)
    ctx = m.Context(model, m.Lora(16, 32.0, m.targets_mask(projs)),
                    m.Run(B, S, base_dtype, int8_in_gemm=args.int8_in_gemm, lm_head_chunk=args.lm_head_chunk,
                          deterministic=args.deterministic),
                    device=local)
    if world > 1:
        uid = share_unique_id(dist_, rank, world, m.Context.dp_unique_id)
        ctx.dp_set_timeout_ms(120000)
        ctx.dp_init(uid, rank, world)
    ctx.init_base_synthetic(seed=1, std=0.02)
    ctx.init_lora_synthetic(seed=2, b_std=0.01)

    tok, tgt = make_tokens(model.vocab, B, S, shard_seed(rank), dist)
    d_tok = torch.from_numpy(tok).cuda()
    d_tgt = torch.from_numpy(tgt).cuda()
    h_tok = torch.from_numpy(tok).pin_memory()
    h_tgt = torch.from_numpy(tgt).pin_memory()
    opt = m.AdamW()
    stream = torch.cuda.ExternalStream(ctx.stream())

    step = 0
    for _ in range(args.warmup):
        step += 1
        ctx.train_step_device(d_tok.data_ptr(), d_tgt.data_ptr(), B, S, opt, step)
    warm_loss = ctx.read_loss()

    # ---------------------------------------------------- timed: device-resident
    barrier()
    torch.cuda.synchronize()
    clocks = ClockSampler(local) if rank == 0 else None
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        step += 1
        ctx.train_step_device(d_tok.data_ptr(), d_tgt.data_ptr(), B, S, opt, step)
    e1.record(stream)
    e1.synchronize()
    torch.cuda.synchronize()
    barrier()
    clk = clocks.stop() if clocks else None
    ms = max_over_ranks(e0.elapsed_time(e1) / args.steps)
    loss = ctx.read_loss()
    tokens_per_step = B * S * world
    value = tokens_per_step / (ms / 1e3)

    # ------------------------------------------------ e2e: host-buffer public API
    # the same number of steps as `value`, timed by the host clock: every call
    # copies this step's tokens/targets from pinned host memory, runs the step
    # and reads the loss back (llmcu_train_step returns after that D2H copy)
    n_e2e = args.steps
    barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(n_e2e):
        step += 1
        ctx.train_step(h_tok.numpy(), h_tgt.numpy(), opt, step)
    t1 = time.perf_counter()
    barrier()
    ms_e2e = max_over_ranks((t1 - t0) * 1e3 / n_e2e)
    e2e = {"value": round(tokens_per_step / (ms_e2e / 1e3), 3), "unit": UNIT,
           "h2d_bytes_per_step": int(h_tok.numel() * 4 + h_tgt.numel() * 4), "d2h_bytes_per_step": 8,
           "ms_per_step": round(ms_e2e, 3), "steps": n_e2e, "timer": "host perf_counter, max over ranks",
           "api": "llmcu_train_step (host int32 tokens/targets; the loss and the device error word, 4 B each, "
                  "read back every step)"}

    # ------------------------------------- per-kernel-class events (roofline)
    n_prof = 2
    barrier()
    ctx.profile_enable(True)
    ctx.profile_read(reset=True)
    for _ in range(n_prof):
        step += 1
        ctx.train_step_device(d_tok.data_ptr(), d_tgt.data_ptr(), B, S, opt, step)
    torch.cuda.synchronize()
    prof = ctx.profile_read(reset=True)
    ctx.profile_enable(False)
    barrier()
    pk = peaks()
    g = prof["gemm_tc"]
    gemm_ms_step = g["ms"] / n_prof
    gemm_launches_step = g["launches"] / n_prof
    alg_flops_step = layer_gemm_flops_per_token(model) * B * S
    per_launch_flops = alg_flops_step / gemm_launches_step
    per_launch_s = gemm_ms_step / gemm_launches_step / 1e3
    achieved = per_launch_flops / per_launch_s / 1e12
    # the lm_head section: vocabulary-streamed logits + cross-entropy + d_xf
    lh = prof.get("lm_head", {"ms": 0.0, "launches": 0})
    lh_ms = lh["ms"] / n_prof
    lh_flops = lm_head_flops_per_token(model) * B * S
    lm_head = {"ms_per_step": round(lh_ms, 3), "launches_per_step": lh["launches"] / n_prof,
               "alg_tflop_per_step": round(lh_flops / 1e12, 3),
               "achieved_tflops": round(lh_flops / (lh_ms / 1e3) / 1e12, 2) if lh_ms > 0 else None,
               "frac_of_sustained": round(lh_flops / (lh_ms / 1e3) / 1e12 / pk["bf16_tflops_sustained"], 4)
               if lh_ms > 0 else None}
    traffic = None
    prof_path = os.path.join(ROOT, "profiles", "gemm_traffic_c2.txt")
    if os.path.exists(prof_path):
        with open(prof_path) as f:
            tr = json.load(f).get(args.workload)
        if tr:
            traffic = tr.get("dram_bytes_per_launch")
    roofline = {"kernel": "gemm_tc_kernel (tcgen05/TMEM, the 28 layers' linear layers)", "bound": "tensor",
                "achieved": round(achieved, 2), "peak": pk["bf16_tflops_sustained"], "unit": "TFLOP/s",
                "frac": round(achieved / pk["bf16_tflops_sustained"], 4), "traffic": traffic,
                "peak_src": f"{pk['src']} sustained bf16 (kernel timed inside a long step)",
                "alg_flops_per_launch": per_launch_flops, "launches_per_step": gemm_launches_step,
                "ms_per_step": round(gemm_ms_step, 3)}
    kernels = {k: {"ms_per_step": round(v["ms"] / n_prof, 3), "launches_per_step": v["launches"] / n_prof}
               for k, v in prof.items() if v["launches"]}
    # compute-stream wait for the allreduces the backward did not hide (events
    # on the compute stream; the adapter gradients run on it in this pass)
    dp_exposed_ms = round(prof.get("dp_exposed", {}).get("ms", 0.0) / n_prof, 3)
    gpu_launches = int(sum(v["launches"] for v in prof.values()) / n_prof * args.steps)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            cpu = cpu_baseline(S if S <= 512 else 512)
        except Exception as exc:  # the baseline must not take the bench down
            cpu = {"value": None, "unit": UNIT, "error": str(exc)[:200]}

    if rank == 0:
        step_alg = algorithmic_flops_per_token(model, S, ctx.lora_param_count()) * tokens_per_step
        line = {
            "metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 3), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f16 operands, f32 accumulate / master weights",
            "data": "synthetic (device-generated N(0,0.02) base, seeded Zipf/uniform token ids)",
            "config": {"workload": args.workload, "description": desc,
                       "model": "qwen3-1.7b-shape" + ("" if args.layers == 28 else f" ({args.layers} layers)"),
                       "global_batch": B * world, "seq_len": S, "parallelism": f"dp{world}",
                       "lora": "rank 16 alpha 32 on " + "/".join(projs),
                       "int8": ("codes staged by the GEMMs" if args.int8_in_gemm else "one dequant pass per weight")
                       if base_dtype else None, "deterministic": bool(args.deterministic),
                       "l2": "inputs larger than L2 (6.9 GB of weights "
                       "and ~9 GB of activations stream per step); no flush"},
            "step_roofline": {"alg_tflop_per_step": round(step_alg / 1e12, 3),
                              "achieved_tflops": round(step_alg / (ms / 1e3) / 1e12 / world, 2),
                              "frac_of_peak_per_gpu": round(step_alg / (ms / 1e3) / 1e12 / world
                                                            / pk["bf16_tflops_sustained"], 4)},
            "roofline": roofline, "lm_head": lm_head, "e2e": e2e, "dp_exposed_ms_per_step": dp_exposed_ms if world > 1 else None, "cpu_baseline": cpu, "gpu_launches": gpu_launches,
            "kernels": kernels, "clocks": clk, "loss": round(loss, 5), "warm_loss": round(warm_loss, 5),
        }
        print(json.dumps(line))
    ctx.close()
    if world > 1:
        dist_.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
