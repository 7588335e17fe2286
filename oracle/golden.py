"""CPU golden for the Qwen3 LoRA training step -- TEST INFRASTRUCTURE ONLY.

This module is the oracle that the CUDA product is checked against.  It is
imported only by ``tests/``, by ``__graft_entry__.smoke()`` and by the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py``; the product
(``libllmcu.so`` and the ``llm_train`` driver) never calls it.

It restates, in torch fp32 autograd on the CPU, the step that llm.cu's
``llm_train`` runs (reference paths are inside the visheshnarayan/llm.cu tree):

* forward order ............ src/kernels/lora_forward.cu:194-304
* RMSNorm  x*rsqrt(mean x^2+eps)*w ........ src/kernels/rmsnorm.cu:30-32
* QK-norm per head (RMSNorm over head_dim) src/kernels/lora_forward.cu:233-234
* RoPE, half-split pairs (d, d+hd/2),
  inv_freq = theta^(-2d/hd) ............... src/kernels/rope.cu:15-35
* causal GQA attention, scale 1/sqrt(hd) .. src/kernels/lora_forward.cu:60-118
* SwiGLU  silu(g)*u ....................... src/kernels/activation.cu:9
* LoRA    y += (alpha/r) * (x A^T) B^T .... src/kernels/lora.cu:190-198
  (the reference adapts q/k/v/o only, include/lora.h:22-27; the same
  formula on gate_proj / up_proj / down_proj when ``make_lora(projs=...)``
  includes them -- a projection without adapter keys gets no LoRA term)
* cross-entropy over positions 0..S-2 of
  each sequence (last position skipped) .. src/kernels/loss.cu:18-69
* AdamW (decoupled weight decay) .......... src/kernels/lora.cu:212-219

Autograd gives the true gradient.  ``ref_bugs=True`` instead reproduces the
four places where the reference's hand-written backward departs from it, so
that the golden can be pinned against the reference's own CUDA build
(oracle/ref_harness):

* the final-RMSNorm backward is evaluated at post_attn[L-1] instead of
  the real pre-norm hidden ............... src/kernels/lora_backward.cu:245-267
* the LoRA dX term reads A ([r, d_in]) as if it were [d_in, r]
  ........................................ src/kernels/lora_backward.cu:87
* the last position gets no dlogits row (its gradient is zero; the
  reference leaves the row uninitialised, the harness zeroes it)
  ........................................ src/kernels/loss.cu:18-21
* the SwiGLU backward runs in place with d_swiglu aliased to d_gate
  (src/kernels/lora_backward.cu:287 calls silu_backward(d_gate, .., d_gate,
  d_up)), so d_up is formed from the already-overwritten d_gate:
  d_up = (dy * u * silu'(g)) * silu(g) instead of dy * silu(g)
  ........................................ src/kernels/activation.cu:35-36

Pinning: with ``ref_bugs=True`` this golden reproduces the reference
trainer's own CUDA build (oracle/ref_harness, compiled from the reference
sources) on seeded inputs -- loss, every LoRA gradient and the post-AdamW
adapters agree to ~2e-6 relative (fixtures tests/golden/ref_tiny_*.npz,
checked by tests/test_oracle.py).  The CUDA product is checked against the
default (true-gradient) mode.
"""
from __future__ import annotations

import dataclasses
import math
from typing import Dict, Optional, Tuple

import numpy as np
import torch

PROJS = ("wq", "wk", "wv", "wo")
# MLP adapters: not in the reference (include/lora.h:22-27 fixes q/k/v/o); the
# same y += s (x A^T) B^T on gate_proj, up_proj and down_proj.
MLP_PROJS = ("w_gate", "w_up", "w_down")
ALL_PROJS = PROJS + MLP_PROJS


@dataclasses.dataclass(frozen=True)
class ModelCfg:
    hidden: int
    n_layers: int
    n_heads: int
    n_kv_heads: int
    head_dim: int
    ffn: int
    vocab: int
    lora_rank: int
    lora_alpha: float
    rope_theta: float = 1.0e6
    rms_eps: float = 1.0e-6

    @property
    def q_dim(self) -> int:
        return self.n_heads * self.head_dim

    @property
    def kv_dim(self) -> int:
        return self.n_kv_heads * self.head_dim

    @property
    def lora_scale(self) -> float:
        return float(self.lora_alpha) / float(self.lora_rank)

    def adapter_dims(self, proj: str) -> Tuple[int, int]:
        """(d_out, d_in) of one adapter, as include/lora.h:22-27 of the reference."""
        return {
            "wq": (self.q_dim, self.hidden),
            "wk": (self.kv_dim, self.hidden),
            "wv": (self.kv_dim, self.hidden),
            "wo": (self.hidden, self.q_dim),
            "w_gate": (self.ffn, self.hidden),
            "w_up": (self.ffn, self.hidden),
            "w_down": (self.hidden, self.ffn),
        }[proj]

    def n_lora_params(self, projs=PROJS) -> int:
        n = 0
        for p in projs:
            d_out, d_in = self.adapter_dims(p)
            n += self.lora_rank * (d_in + d_out)
        return n * self.n_layers


# BASELINE.json configs[0] (tiny) and configs[1..4] (Qwen3-1.7B shape).
CFG_TINY = ModelCfg(hidden=256, n_layers=2, n_heads=4, n_kv_heads=2, head_dim=64,
                    ffn=768, vocab=4096, lora_rank=4, lora_alpha=8.0)
CFG_QWEN3_1P7B = ModelCfg(hidden=2048, n_layers=28, n_heads=16, n_kv_heads=8,
                          head_dim=128, ffn=6144, vocab=151936, lora_rank=16,
                          lora_alpha=32.0)


def layer_slice(cfg: ModelCfg, n_layers: int, vocab: Optional[int] = None) -> ModelCfg:
    """The same architecture with fewer layers (and optionally a smaller vocab)."""
    return dataclasses.replace(cfg, n_layers=n_layers, vocab=vocab or cfg.vocab)


# ----------------------------------------------------------------------------
# seeded synthetic inputs (numpy PCG64)
# ----------------------------------------------------------------------------

def make_base_weights(cfg: ModelCfg, seed: int, std: float = 0.02,
                      round_fp16: bool = False) -> Dict[str, np.ndarray]:
    """Frozen base weights ~ N(0, std) in fp32, norm gains 1 (configs[0..4]).

    Keys follow the reference's weight files (src/train.cu:56-89):
    ``embed``, ``final_norm`` and ``L{l}.{attn_norm,ffn_norm,wq,wk,wv,wo,q_norm,
    k_norm,w_gate,w_up,w_down}``.  The lm_head is tied to ``embed``.
    """
    rng = np.random.Generator(np.random.PCG64(seed))
    H, Q, KV, I, V, hd = cfg.hidden, cfg.q_dim, cfg.kv_dim, cfg.ffn, cfg.vocab, cfg.head_dim

    def draw(*shape):
        w = rng.standard_normal(size=shape, dtype=np.float32) * np.float32(std)
        if round_fp16:
            w = w.astype(np.float16).astype(np.float32)
        return w

    w: Dict[str, np.ndarray] = {"embed": draw(V, H), "final_norm": np.ones(H, np.float32)}
    for l in range(cfg.n_layers):
        p = f"L{l}."
        w[p + "attn_norm"] = np.ones(H, np.float32)
        w[p + "ffn_norm"] = np.ones(H, np.float32)
        w[p + "wq"] = draw(Q, H)
        w[p + "wk"] = draw(KV, H)
        w[p + "wv"] = draw(KV, H)
        w[p + "wo"] = draw(H, Q)
        w[p + "q_norm"] = np.ones(hd, np.float32)
        w[p + "k_norm"] = np.ones(hd, np.float32)
        w[p + "w_gate"] = draw(I, H)
        w[p + "w_up"] = draw(I, H)
        w[p + "w_down"] = draw(H, I)
    return w


def make_lora(cfg: ModelCfg, seed: int, b_std: float = 0.01, projs=PROJS) -> Dict[str, np.ndarray]:
    """LoRA adapters: A ~ U(+-1/sqrt(in)) [r, in], B ~ N(0, b_std) [out, r],
    for the projections ``projs`` (default: the reference's q/k/v/o)."""
    rng = np.random.Generator(np.random.PCG64(seed))
    out: Dict[str, np.ndarray] = {}
    r = cfg.lora_rank
    for l in range(cfg.n_layers):
        for p in projs:
            d_out, d_in = cfg.adapter_dims(p)
            bound = 1.0 / math.sqrt(d_in)
            out[f"L{l}.{p}.A"] = rng.uniform(-bound, bound, size=(r, d_in)).astype(np.float32)
            out[f"L{l}.{p}.B"] = (rng.standard_normal(size=(d_out, r), dtype=np.float32)
                                  * np.float32(b_std))
    return out


def make_tokens(cfg: ModelCfg, batch: int, seq: int, seed: int,
                dist: str = "uniform", zipf_s: float = 1.1) -> Tuple[np.ndarray, np.ndarray]:
    """(inputs, targets) int32 [batch, seq]; targets are the inputs shifted by one.

    ``dist='zipf'`` draws a truncated Zipf by rank, p(k) ~ k^-s for k=1..V, with
    the identity rank->id map (id = k-1).
    """
    rng = np.random.Generator(np.random.PCG64(seed))
    n = batch * (seq + 1)
    if dist == "uniform":
        ids = rng.integers(0, cfg.vocab, size=n, dtype=np.int64)
    elif dist == "zipf":
        k = np.arange(1, cfg.vocab + 1, dtype=np.float64)
        p = k ** (-zipf_s)
        cdf = np.cumsum(p)
        cdf /= cdf[-1]
        ids = np.searchsorted(cdf, rng.random(n), side="right")
        ids = np.minimum(ids, cfg.vocab - 1)
    else:
        raise ValueError(dist)
    win = ids.reshape(batch, seq + 1).astype(np.int32)
    return np.ascontiguousarray(win[:, :seq]), np.ascontiguousarray(win[:, 1:])


# ----------------------------------------------------------------------------
# model pieces
# ----------------------------------------------------------------------------

def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """x * rsqrt(mean(x^2) + eps) * w over the last dim (src/kernels/rmsnorm.cu:30-32)."""
    return x * torch.rsqrt((x * x).mean(-1, keepdim=True) + eps) * w


def rmsnorm_backward_at(dy: torch.Tensor, x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """dx of RMSNorm evaluated at x (src/kernels/rmsnorm.cu:53-90): r*(dy*w - c*x)."""
    n = x.shape[-1]
    r = torch.rsqrt((x * x).mean(-1, keepdim=True) + eps)
    c = (r * r / n) * (dy * w * x).sum(-1, keepdim=True)
    return r * (dy * w - c * x)


class _FinalNormRefBug(torch.autograd.Function):
    """Final RMSNorm whose backward is evaluated at a stand-in input (post_attn[L-1])."""

    @staticmethod
    def forward(ctx, x, x_bwd, w, eps):
        ctx.save_for_backward(x_bwd, w)
        ctx.eps = eps
        return rmsnorm(x, w, eps)

    @staticmethod
    def backward(ctx, dy):
        x_bwd, w = ctx.saved_tensors
        return rmsnorm_backward_at(dy, x_bwd, w, ctx.eps), None, None, None


class _SwiGLURefBug(torch.autograd.Function):
    """silu(g) * u whose backward reproduces the reference's in-place d_gate / d_swiglu aliasing."""

    @staticmethod
    def forward(ctx, g, u):
        ctx.save_for_backward(g, u)
        return torch.nn.functional.silu(g) * u

    @staticmethod
    def backward(ctx, dy):
        g, u = ctx.saved_tensors
        sig = torch.sigmoid(g)
        silu = g * sig
        dg = dy * u * (sig * (1.0 + g * (1.0 - sig)))
        du = dg * silu                              # reads the overwritten d_gate
        return dg, du


class _LoraDownRefBug(torch.autograd.Function):
    """h = x A^T whose dX reads A [r, d_in] with a [d_in, r] layout (the reference's misread)."""

    @staticmethod
    def forward(ctx, x, A):
        ctx.save_for_backward(x, A)
        return x @ A.t()

    @staticmethod
    def backward(ctx, dh):
        x, A = ctx.saved_tensors
        r, d_in = A.shape
        a_misread = A.reshape(d_in, r)            # A_flat[n*r + k] used as A[k, n]
        dx = dh @ a_misread.t()
        dA = dh.reshape(-1, r).t() @ x.reshape(-1, d_in)
        return dx, dA


def rope_tables(cfg: ModelCfg, seq: int) -> Tuple[torch.Tensor, torch.Tensor]:
    """cos/sin [seq, hd/2] with inv_freq = 1/theta^(2d/hd), angle = pos*inv_freq in fp32."""
    half = cfg.head_dim // 2
    d = torch.arange(half, dtype=torch.float32)
    inv = 1.0 / torch.pow(torch.tensor(cfg.rope_theta, dtype=torch.float32), (2.0 * d) / cfg.head_dim)
    ang = torch.arange(seq, dtype=torch.float32)[:, None] * inv[None, :]
    return torch.cos(ang), torch.sin(ang)


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """x [B, S, nh, hd]; pairs (d, d+hd/2) rotated by angle (src/kernels/rope.cu:26-35)."""
    half = x.shape[-1] // 2
    x0, x1 = x[..., :half], x[..., half:]
    c = cos[None, :, None, :]
    s = sin[None, :, None, :]
    return torch.cat([x0 * c - x1 * s, x1 * c + x0 * s], dim=-1)


def causal_gqa_attention(q, k, v, scale):
    """q [B,S,nq,hd], k/v [B,S,nkv,hd] -> [B,S,nq,hd]; causal softmax(q k^T * scale) v."""
    B, S, nq, hd = q.shape
    nkv = k.shape[2]
    g = nq // nkv
    k = k.repeat_interleave(g, dim=2)
    v = v.repeat_interleave(g, dim=2)
    qh, kh, vh = q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)
    s = (qh @ kh.transpose(-1, -2)) * scale
    mask = torch.ones(S, S, dtype=torch.bool).triu(1)
    s = s.masked_fill(mask, float("-inf"))
    p = torch.softmax(s, dim=-1)
    return (p @ vh).transpose(1, 2)


# ----------------------------------------------------------------------------
# one step
# ----------------------------------------------------------------------------

def _layers(cfg: ModelCfg, W: Dict[str, torch.Tensor], lora_add, tokens: np.ndarray, cos, sin,
            ref_bugs: bool = False):
    """Embedding and every layer (src/kernels/lora_forward.cu:194-304): the
    pre-final-norm hidden [B, S, H] and the last layer's post-attention hidden."""
    B, S = tokens.shape
    H, hd, nq, nkv = cfg.hidden, cfg.head_dim, cfg.n_heads, cfg.n_kv_heads
    eps = cfg.rms_eps
    x = W["embed"][torch.from_numpy(tokens.astype(np.int64))]   # [B,S,H]
    post_attn_last = None
    for l in range(cfg.n_layers):
        p = f"L{l}."
        xn = rmsnorm(x, W[p + "attn_norm"], eps)
        q = xn @ W[p + "wq"].t() + lora_add(xn, p + "wq")
        k = xn @ W[p + "wk"].t() + lora_add(xn, p + "wk")
        v = xn @ W[p + "wv"].t() + lora_add(xn, p + "wv")
        q = rmsnorm(q.view(B, S, nq, hd), W[p + "q_norm"], eps)
        k = rmsnorm(k.view(B, S, nkv, hd), W[p + "k_norm"], eps)
        q = apply_rope(q, cos, sin)
        k = apply_rope(k, cos, sin)
        o = causal_gqa_attention(q, k, v.view(B, S, nkv, hd), 1.0 / math.sqrt(hd))
        o = o.reshape(B, S, nq * hd)
        x = x + o @ W[p + "wo"].t() + lora_add(o, p + "wo")
        post_attn_last = x
        xn2 = rmsnorm(x, W[p + "ffn_norm"], eps)
        g = xn2 @ W[p + "w_gate"].t() + lora_add(xn2, p + "w_gate")
        u = xn2 @ W[p + "w_up"].t() + lora_add(xn2, p + "w_up")
        act = _SwiGLURefBug.apply(g, u) if ref_bugs else torch.nn.functional.silu(g) * u
        x = x + act @ W[p + "w_down"].t() + lora_add(act, p + "w_down")
    return x, post_attn_last


def forward_logits(cfg: ModelCfg, base: Dict[str, np.ndarray], lora: Dict[str, np.ndarray],
                   tokens: np.ndarray) -> np.ndarray:
    """Logits [B, S, V] of the forward (fp32, no gradient) -- what the
    reference's inference path computes position by position
    (src/kernels/forward.cu:340-394)."""
    T = lambda a: torch.from_numpy(np.ascontiguousarray(a))
    W = {k: T(v) for k, v in base.items()}
    A = {k: T(v) for k, v in lora.items()}
    s_lora = cfg.lora_scale
    def lora_add(x, name):  # 0 for a projection without an adapter
        if name + ".A" not in A:
            return 0.0
        return ((x @ A[name + ".A"].t()) @ A[name + ".B"].t()) * s_lora
    cos, sin = rope_tables(cfg, tokens.shape[1])
    with torch.no_grad():
        x, _ = _layers(cfg, W, lora_add, tokens, cos, sin)
        return (rmsnorm(x, W["final_norm"], cfg.rms_eps) @ W["embed"].t()).numpy()


def generate_greedy(cfg: ModelCfg, base, lora, prompt: np.ndarray, n_new: int):
    """Greedy continuation (first maximum on ties, as llm_engine's host loop,
    src/main.cu:362-366): (tokens [n_new], logits [n_new, V]), each step
    re-running the forward over the whole prefix."""
    seq = [int(t) for t in np.asarray(prompt).reshape(-1)]
    toks, logits = [], []
    for _ in range(n_new):
        lg = forward_logits(cfg, base, lora, np.array([seq], dtype=np.int32))[0, -1]
        t = int(np.argmax(lg))
        toks.append(t)
        logits.append(lg)
        seq.append(t)
    return np.array(toks, dtype=np.int32), np.stack(logits)


@dataclasses.dataclass
class StepResult:
    loss: float
    grads: Dict[str, np.ndarray]          # "L{l}.{proj}.{A,B}" -> fp32 gradient
    n_positions: int


def forward_backward(cfg: ModelCfg, base: Dict[str, np.ndarray], lora: Dict[str, np.ndarray],
                     tokens: np.ndarray, targets: np.ndarray, *, ref_bugs: bool = False,
                     all_positions: bool = False, threads: Optional[int] = None) -> StepResult:
    """Loss (mean NLL) and LoRA gradients for one batch [B, S].

    Default loss convention = the reference's: mean over positions 0..S-2 of
    every sequence (src/kernels/loss.cu:18-21,74-91).  ``all_positions`` uses
    every position instead.
    """
    if threads:
        torch.set_num_threads(threads)
    B, S = tokens.shape
    H, hd, nq, nkv = cfg.hidden, cfg.head_dim, cfg.n_heads, cfg.n_kv_heads
    eps = cfg.rms_eps
    s_lora = cfg.lora_scale
    T = lambda a: torch.from_numpy(np.ascontiguousarray(a))

    params: Dict[str, torch.Tensor] = {k: T(v).clone().requires_grad_(True) for k, v in lora.items()}
    W = {k: T(v) for k, v in base.items()}
    E = W["embed"]
    cos, sin = rope_tables(cfg, S)

    def lora_add(x, name):
        if name + ".A" not in params:  # a projection without an adapter
            return 0.0
        A, Bm = params[name + ".A"], params[name + ".B"]
        h = _LoraDownRefBug.apply(x, A) if ref_bugs else x @ A.t()
        return (h @ Bm.t()) * s_lora

    with torch.enable_grad():
        x, post_attn_last = _layers(cfg, W, lora_add, tokens, cos, sin, ref_bugs)
        if ref_bugs:
            xf = _FinalNormRefBug.apply(x, post_attn_last.detach(), W["final_norm"], eps)
        else:
            xf = rmsnorm(x, W["final_norm"], eps)
        logits = xf @ E.t()                                       # [B,S,V]
        tgt = torch.from_numpy(targets.astype(np.int64))
        if all_positions:
            lg, tg = logits.reshape(-1, cfg.vocab), tgt.reshape(-1)
        else:
            lg, tg = logits[:, : S - 1].reshape(-1, cfg.vocab), tgt[:, : S - 1].reshape(-1)
        n_pos = int(tg.numel())
        loss = torch.nn.functional.cross_entropy(lg, tg, reduction="mean")
        loss.backward()
    grads = {k: v.grad.detach().numpy().copy() for k, v in params.items()}
    return StepResult(loss=float(loss.detach()), grads=grads, n_positions=n_pos)


def adamw(lora: Dict[str, np.ndarray], grads: Dict[str, np.ndarray],
          m: Dict[str, np.ndarray], v: Dict[str, np.ndarray], *, lr: float, beta1: float,
          beta2: float, eps: float, wd: float, step: int) -> None:
    """In-place AdamW in fp32, term by term as src/kernels/lora.cu:206-246."""
    f = np.float32
    bc1 = f(1.0) - f(beta1) ** f(step)
    bc2 = f(1.0) - f(beta2) ** f(step)
    for k in lora:
        g = grads[k].astype(np.float32)
        mi = f(beta1) * m[k] + (f(1.0) - f(beta1)) * g
        vi = f(beta2) * v[k] + (f(1.0) - f(beta2)) * g * g
        m[k][...] = mi
        v[k][...] = vi
        m_hat = mi / bc1
        v_hat = vi / bc2
        lora[k][...] = lora[k] * (f(1.0) - f(lr) * f(wd)) - f(lr) * m_hat / (np.sqrt(v_hat) + f(eps))


def train_step(cfg: ModelCfg, base, lora, m, v, tokens, targets, *, lr=3e-4, beta1=0.9,
               beta2=0.999, eps=1e-8, wd=0.01, step=1, **kw) -> StepResult:
    """forward + backward + AdamW; updates ``lora``, ``m``, ``v`` in place."""
    res = forward_backward(cfg, base, lora, tokens, targets, **kw)
    adamw(lora, res.grads, m, v, lr=lr, beta1=beta1, beta2=beta2, eps=eps, wd=wd, step=step)
    return res


def zeros_like_lora(lora: Dict[str, np.ndarray]) -> Dict[str, np.ndarray]:
    return {k: np.zeros_like(a) for k, a in lora.items()}


def algorithmic_flops_per_token(cfg: ModelCfg, seq: int, projs=PROJS) -> float:
    """4*N_lin + 3*(2*S*hd*nq*L) + 6*n_lora (forward + dX, causal attention, LoRA)."""
    per_layer = (cfg.q_dim * cfg.hidden + 2 * cfg.kv_dim * cfg.hidden + cfg.hidden * cfg.q_dim
                 + 3 * cfg.ffn * cfg.hidden)
    n_lin = cfg.n_layers * per_layer + cfg.vocab * cfg.hidden
    attn = 3 * (2 * seq * cfg.head_dim * cfg.n_heads * cfg.n_layers)
    return float(4 * n_lin + attn + 6 * cfg.n_lora_params(projs))


def rel_l2(a: np.ndarray, b: np.ndarray) -> float:
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def cosine(a: np.ndarray, b: np.ndarray) -> float:
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(a @ b / max(np.linalg.norm(a) * np.linalg.norm(b), 1e-300))
