"""File format between the parity tests and oracle/ref_harness (the reference
trainer's own CUDA code).  TEST INFRASTRUCTURE ONLY.

Input  (little-endian): int32 dims[8] = hidden, layers, heads, kv_heads,
head_dim, ffn, vocab, rank; int32 batch, seq; int32 tokens[B*S];
int32 targets[B*S]; float32 adamw[5] = lr, beta1, beta2, eps, wd; then fp32
weights (embed, final_norm, per layer attn_norm ffn_norm wq wk wv wo q_norm
k_norm w_gate w_up w_down); then per layer and projection (wq wk wv wo) the
adapter A [r, d_in] and B [d_out, r].

Output: float32 losses[B]; per layer/projection dA, dB (batch-mean
gradients); per layer/projection A, B after one AdamW step.
"""
from __future__ import annotations

import numpy as np

PROJS = ("wq", "wk", "wv", "wo")
LAYER_KEYS = ("attn_norm", "ffn_norm", "wq", "wk", "wv", "wo", "q_norm", "k_norm", "w_gate", "w_up", "w_down")


def write_input(path, cfg, base, lora, tokens, targets, adamw=(3e-4, 0.9, 0.999, 1e-8, 0.01)):
    B, S = tokens.shape
    with open(path, "wb") as f:
        np.array([cfg.hidden, cfg.n_layers, cfg.n_heads, cfg.n_kv_heads, cfg.head_dim, cfg.ffn, cfg.vocab,
                  cfg.lora_rank, B, S], np.int32).tofile(f)
        np.ascontiguousarray(tokens, np.int32).tofile(f)
        np.ascontiguousarray(targets, np.int32).tofile(f)
        np.array(adamw, np.float32).tofile(f)
        base["embed"].astype(np.float32).tofile(f)
        base["final_norm"].astype(np.float32).tofile(f)
        for l in range(cfg.n_layers):
            for k in LAYER_KEYS:
                base[f"L{l}.{k}"].astype(np.float32).tofile(f)
        for l in range(cfg.n_layers):
            for p in PROJS:
                lora[f"L{l}.{p}.A"].astype(np.float32).tofile(f)
                lora[f"L{l}.{p}.B"].astype(np.float32).tofile(f)


def read_output(path, cfg, batch):
    data = np.fromfile(path, dtype=np.float32)
    off = 0

    def take(n):
        nonlocal off
        out = data[off:off + n]
        off += n
        return out

    losses = take(batch).copy()
    grads, after = {}, {}
    for dst in (grads, after):
        for l in range(cfg.n_layers):
            for p in PROJS:
                d_out, d_in = cfg.adapter_dims(p)
                dst[f"L{l}.{p}.A"] = take(cfg.lora_rank * d_in).reshape(cfg.lora_rank, d_in).copy()
                dst[f"L{l}.{p}.B"] = take(d_out * cfg.lora_rank).reshape(d_out, cfg.lora_rank).copy()
    assert off == data.size, (off, data.size)
    return losses, grads, after
