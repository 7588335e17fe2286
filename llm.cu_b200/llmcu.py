"""ctypes binding of libllmcu.so (include/llmcu.h) for Python callers.

This is the Python-side mirror of the C ABI -- the binding a maintainer of
llm.cu would add to drive the step from Python.  It holds no compute: every
call goes straight to the CUDA library, and importing it fails loudly when the
shared library is missing (there is no CPU fallback).

    from llmcu import Model, Lora, Run, Context, AdamW
    ctx = Context(Model.qwen3_1p7b(), Lora(16, 32.0), Run(max_batch=8, max_seq=512))
    ctx.init_base_synthetic(seed=1); ctx.init_lora_synthetic(seed=2)
    loss = ctx.train_step(tokens, targets, AdamW(), step=1)
"""
from __future__ import annotations

import ctypes as C
import os
from dataclasses import dataclass
from typing import Optional

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("LLMCU_LIB", os.path.join(_HERE, "libllmcu.so"))

OK = 0
STATUS = {0: "OK", 1: "INVALID_ARG", 2: "CUDA", 3: "OOM", 4: "IO", 5: "NCCL", 6: "TIMEOUT",
          7: "DEVICE_CHECK", 8: "UNSUPPORTED"}

T_EMBED, T_FINAL_NORM, T_ATTN_NORM, T_FFN_NORM, T_WQ, T_WK, T_WV, T_WO, T_Q_NORM, T_K_NORM, \
    T_W_GATE, T_W_UP, T_W_DOWN = range(13)
P_Q, P_K, P_V, P_O, P_GATE, P_UP, P_DOWN = range(7)
TARGETS_ATTN, TARGETS_MLP, TARGETS_ALL = 0x0F, 0x70, 0x7F
# adapter names (golden dict keys and lora_step file names), by projection id
PROJ_NAMES = {P_Q: "wq", P_K: "wk", P_V: "wv", P_O: "wo", P_GATE: "w_gate", P_UP: "w_up", P_DOWN: "w_down"}


def targets_mask(names) -> int:
    """Target mask of an iterable of adapter names ("wq", ..., "w_down")."""
    ids = {n: p for p, n in PROJ_NAMES.items()}
    m = 0
    for n in names:
        m |= 1 << ids[n]
    return m
BASE_FP16, BASE_INT8 = 0, 1


class LlmcuError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"llmcu status {status} ({STATUS.get(status, '?')}): {msg}")
        self.status = status


class _ModelCfg(C.Structure):
    _fields_ = [("hidden", C.c_int32), ("n_layers", C.c_int32), ("n_heads", C.c_int32),
                ("n_kv_heads", C.c_int32), ("head_dim", C.c_int32), ("ffn", C.c_int32),
                ("vocab", C.c_int32), ("rope_theta", C.c_float), ("rms_eps", C.c_float)]


class _LoraCfg(C.Structure):
    _fields_ = [("rank", C.c_int32), ("alpha", C.c_float), ("targets", C.c_int32)]


class _RunCfg(C.Structure):
    _fields_ = [("max_batch", C.c_int32), ("max_seq", C.c_int32), ("base_dtype", C.c_int32),
                ("loss_all_positions", C.c_int32), ("int8_in_gemm", C.c_int32), ("lm_head_chunk", C.c_int32),
                ("deterministic", C.c_int32)]


class _LoraLayout(C.Structure):
    _fields_ = [("n_layers", C.c_int32), ("hidden", C.c_int32), ("q_dim", C.c_int32), ("kv_dim", C.c_int32),
                ("ffn", C.c_int32), ("rank", C.c_int32), ("targets", C.c_int32)]


class _AdamWCfg(C.Structure):
    _fields_ = [("lr", C.c_float), ("beta1", C.c_float), ("beta2", C.c_float), ("eps", C.c_float),
                ("weight_decay", C.c_float)]


@dataclass(frozen=True)
class Model:
    hidden: int
    n_layers: int
    n_heads: int
    n_kv_heads: int
    head_dim: int
    ffn: int
    vocab: int
    rope_theta: float = 1.0e6
    rms_eps: float = 1.0e-6

    @staticmethod
    def tiny() -> "Model":
        return Model(256, 2, 4, 2, 64, 768, 4096)

    @staticmethod
    def qwen3_1p7b(n_layers: int = 28, vocab: int = 151936) -> "Model":
        return Model(2048, n_layers, 16, 8, 128, 6144, vocab)


@dataclass(frozen=True)
class Lora:
    rank: int = 16
    alpha: float = 32.0
    targets: int = TARGETS_ATTN  # llmcu_lora_cfg.targets: bit p = projection p has an adapter

    def projs(self):
        return [p for p in PROJ_NAMES if (self.targets >> p) & 1]


@dataclass(frozen=True)
class Run:
    max_batch: int = 1
    max_seq: int = 512
    base_dtype: int = BASE_FP16
    loss_all_positions: bool = False
    int8_in_gemm: bool = False  # INT8 base: the GEMMs stage the codes themselves (else one dequant pass per weight)
    lm_head_chunk: int = 0      # vocabulary columns per lm_head chunk (multiple of 256); 0 = automatic
    deterministic: bool = False  # fixed-order sums everywhere (dQ slabs): bit-identical repeated steps


@dataclass(frozen=True)
class AdamW:
    lr: float = 3e-4
    beta1: float = 0.9
    beta2: float = 0.999
    eps: float = 1e-8
    weight_decay: float = 0.01


_lib: Optional[C.CDLL] = None

_SIGS = {
    "llmcu_version": (C.c_char_p, []),
    "llmcu_last_error": (C.c_char_p, [C.c_void_p]),
    "llmcu_device_bytes": (C.c_size_t, [C.c_void_p]),
    "llmcu_stream": (C.c_void_p, [C.c_void_p]),
    "llmcu_lora_param_count": (C.c_int64, [C.c_void_p]),
    "llmcu_lora_targets": (C.c_int32, [C.c_void_p]),
    "llmcu_ctx_create": (C.c_int, [C.POINTER(_ModelCfg), C.POINTER(_LoraCfg), C.POINTER(_RunCfg), C.c_int,
                                   C.POINTER(C.c_void_p)]),
    "llmcu_ctx_destroy": (None, [C.c_void_p]),
    "llmcu_synchronize": (C.c_int, [C.c_void_p]),
    "llmcu_set_base_tensor": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_void_p]),
    "llmcu_load_base_fp32_files": (C.c_int, [C.c_void_p, C.c_char_p]),
    "llmcu_init_base_synthetic": (C.c_int, [C.c_void_p, C.c_uint64, C.c_float]),
    "llmcu_set_lora": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_void_p]),
    "llmcu_get_lora": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_void_p]),
    "llmcu_get_lora_grads": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_void_p]),
    "llmcu_init_lora_synthetic": (C.c_int, [C.c_void_p, C.c_uint64, C.c_float]),
    "llmcu_reset_optimizer": (C.c_int, [C.c_void_p]),
    "llmcu_train_step": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.POINTER(_AdamWCfg),
                                   C.c_int, C.POINTER(C.c_float)]),
    "llmcu_train_step_device": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int,
                                          C.POINTER(_AdamWCfg), C.c_int]),
    "llmcu_read_loss": (C.c_int, [C.c_void_p, C.POINTER(C.c_float)]),
    "llmcu_forward_backward": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int,
                                         C.POINTER(C.c_float)]),
    "llmcu_adamw": (C.c_int, [C.c_void_p, C.POINTER(_AdamWCfg), C.c_int]),
    "llmcu_save_lora": (C.c_int, [C.c_void_p, C.c_char_p, C.c_int]),
    "llmcu_load_lora": (C.c_int, [C.c_void_p, C.c_char_p, C.c_int]),
    "llmcu_save_adamw_state": (C.c_int, [C.c_void_p, C.c_char_p, C.c_int]),
    "llmcu_generate": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.POINTER(C.c_int),
                                 C.c_void_p, C.POINTER(C.c_float)]),
    "llmcu_load_adamw_state": (C.c_int, [C.c_void_p, C.c_char_p, C.c_int]),
    "llmcu_quantize_int8_rows": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p]),
    "llmcu_dp_get_unique_id": (C.c_int, [C.c_void_p]),
    "llmcu_dp_init": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_int]),
    "llmcu_dp_set_timeout_ms": (C.c_int, [C.c_void_p, C.c_int]),
    "llmcu_profile_enable": (C.c_int, [C.c_void_p, C.c_int]),
    "llmcu_profile_read": (C.c_int, [C.c_void_p, C.c_char_p, C.c_size_t, C.c_int]),
    "llmcu_gemm_nt_f16": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int,
                                    C.c_int, C.c_int, C.c_void_p]),
    "llmcu_gemm_nn_f16": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int,
                                    C.c_int, C.c_int, C.c_void_p]),
    "llmcu_attention_fwd": (C.c_int, [C.c_void_p] * 5 + [C.c_int] * 8 + [C.c_void_p]),
    "llmcu_attention_bwd": (C.c_int, [C.c_void_p] * 10 + [C.c_int] * 9 + [C.c_void_p]),
    "llmcu_attention_bwd_noalloc": (C.c_int, [C.c_void_p] * 9 + [C.c_int] * 9 + [C.c_void_p]),
    "llmcu_kernel_checks": (C.c_int, [C.c_void_p, C.POINTER(C.c_int)]),
    "llmcu_kernel_wait_selftest": (C.c_int, [C.c_void_p]),
    "llmcu_lora_layout_count": (C.c_int64, [C.POINTER(_LoraLayout)]),
    "llmcu_lora_files_write": (C.c_int, [C.POINTER(_LoraLayout), C.c_void_p, C.c_char_p, C.c_int]),
    "llmcu_lora_files_read": (C.c_int, [C.POINTER(_LoraLayout), C.c_void_p, C.c_char_p, C.c_int]),
}


def lib() -> C.CDLL:
    """Load libllmcu.so once; raises if it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise FileNotFoundError(f"{LIB_PATH} is missing: build it with `make -C llm.cu_b200`")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def exported_symbols():
    return list(_SIGS)


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(C.c_void_p)


class Context:
    """One training context on one GPU (llmcu_ctx)."""

    def __init__(self, model: Model, lora: Lora, run: Run, device: int = 0):
        L = lib()
        self.model, self.lora, self.run = model, lora, run
        mc = _ModelCfg(model.hidden, model.n_layers, model.n_heads, model.n_kv_heads, model.head_dim,
                       model.ffn, model.vocab, model.rope_theta, model.rms_eps)
        lc = _LoraCfg(lora.rank, lora.alpha, lora.targets)
        rc = _RunCfg(run.max_batch, run.max_seq, run.base_dtype, int(run.loss_all_positions), int(run.int8_in_gemm),
                     int(run.lm_head_chunk), int(run.deterministic))
        h = C.c_void_p()
        st = L.llmcu_ctx_create(C.byref(mc), C.byref(lc), C.byref(rc), device, C.byref(h))
        if st != OK:
            raise LlmcuError(st, "llmcu_ctx_create")
        self._h = h

    # -- plumbing
    def _check(self, st: int, what: str):
        if st != OK:
            raise LlmcuError(st, f"{what}: {lib().llmcu_last_error(self._h).decode()}")

    def close(self):
        if getattr(self, "_h", None):
            lib().llmcu_ctx_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    @property
    def handle(self):
        return self._h

    def device_bytes(self) -> int:
        return int(lib().llmcu_device_bytes(self._h))

    def stream(self) -> int:
        return int(lib().llmcu_stream(self._h) or 0)

    def lora_param_count(self) -> int:
        return int(lib().llmcu_lora_param_count(self._h))

    def lora_targets(self) -> int:
        return int(lib().llmcu_lora_targets(self._h))

    def synchronize(self):
        self._check(lib().llmcu_synchronize(self._h), "synchronize")

    # -- weights
    def set_base_tensor(self, tid: int, layer: int, w: np.ndarray):
        a = np.ascontiguousarray(w, dtype=np.float32)
        self._check(lib().llmcu_set_base_tensor(self._h, tid, layer, _ptr(a)), f"set_base_tensor({tid},{layer})")

    def set_base(self, base: dict):
        """Upload a golden-style dict (keys 'embed', 'final_norm', 'L{l}.wq', ...)."""
        names = {"attn_norm": T_ATTN_NORM, "ffn_norm": T_FFN_NORM, "wq": T_WQ, "wk": T_WK, "wv": T_WV,
                 "wo": T_WO, "q_norm": T_Q_NORM, "k_norm": T_K_NORM, "w_gate": T_W_GATE, "w_up": T_W_UP,
                 "w_down": T_W_DOWN}
        self.set_base_tensor(T_EMBED, 0, base["embed"])
        self.set_base_tensor(T_FINAL_NORM, 0, base["final_norm"])
        for key, arr in base.items():
            if key.startswith("L"):
                l, n = key[1:].split(".", 1)
                self.set_base_tensor(names[n], int(l), arr)

    def load_base_files(self, directory: str):
        self._check(lib().llmcu_load_base_fp32_files(self._h, directory.encode()), "load_base_fp32_files")

    def init_base_synthetic(self, seed: int = 1, std: float = 0.02):
        self._check(lib().llmcu_init_base_synthetic(self._h, seed, std), "init_base_synthetic")

    # -- adapters
    def _dims(self, proj: int):
        m = self.model
        q, kv = m.n_heads * m.head_dim, m.n_kv_heads * m.head_dim
        d_out = {P_Q: q, P_K: kv, P_V: kv, P_O: m.hidden, P_GATE: m.ffn, P_UP: m.ffn, P_DOWN: m.hidden}[proj]
        d_in = {P_O: q, P_DOWN: m.ffn}.get(proj, m.hidden)
        return d_out, d_in

    def set_lora(self, layer: int, proj: int, A: np.ndarray, B: np.ndarray):
        a = np.ascontiguousarray(A, dtype=np.float32)
        b = np.ascontiguousarray(B, dtype=np.float32)
        d_out, d_in = self._dims(proj)
        assert a.shape == (self.lora.rank, d_in) and b.shape == (d_out, self.lora.rank)
        self._check(lib().llmcu_set_lora(self._h, layer, proj, _ptr(a), _ptr(b)), "set_lora")

    def set_lora_dict(self, lora: dict):
        for l in range(self.model.n_layers):
            for i in self.lora.projs():
                p = PROJ_NAMES[i]
                self.set_lora(l, i, lora[f"L{l}.{p}.A"], lora[f"L{l}.{p}.B"])

    def _get_pair(self, fn, layer, proj):
        d_out, d_in = self._dims(proj)
        a = np.empty((self.lora.rank, d_in), np.float32)
        b = np.empty((d_out, self.lora.rank), np.float32)
        self._check(fn(self._h, layer, proj, _ptr(a), _ptr(b)), fn.__name__)
        return a, b

    def get_lora(self, layer: int, proj: int):
        return self._get_pair(lib().llmcu_get_lora, layer, proj)

    def get_lora_grads(self, layer: int, proj: int):
        return self._get_pair(lib().llmcu_get_lora_grads, layer, proj)

    def _dict(self, getter):
        out = {}
        for l in range(self.model.n_layers):
            for p in self.lora.projs():
                n = PROJ_NAMES[p]
                a, b = getter(l, p)
                out[f"L{l}.{n}.A"], out[f"L{l}.{n}.B"] = a, b
        return out

    def lora_dict(self):
        return self._dict(self.get_lora)

    def grads_dict(self):
        return self._dict(self.get_lora_grads)

    def init_lora_synthetic(self, seed: int = 2, b_std: float = 0.01):
        self._check(lib().llmcu_init_lora_synthetic(self._h, seed, b_std), "init_lora_synthetic")

    def reset_optimizer(self):
        self._check(lib().llmcu_reset_optimizer(self._h), "reset_optimizer")

    # -- steps
    @staticmethod
    def _tok(a):
        return np.ascontiguousarray(a, dtype=np.int32)

    @classmethod
    def _batch(cls, tokens, targets):
        """int32 [B, S] tokens and targets of one shape (the library copies
        B * S ids from each host pointer)."""
        t, g = cls._tok(tokens), cls._tok(targets)
        if t.ndim != 2 or g.shape != t.shape:
            raise ValueError(f"tokens {t.shape} and targets {g.shape} must be one [batch, seq] shape")
        return t, g

    def forward_backward(self, tokens: np.ndarray, targets: np.ndarray) -> float:
        t, g = self._batch(tokens, targets)
        B, S = t.shape
        loss = C.c_float()
        self._check(lib().llmcu_forward_backward(self._h, _ptr(t), _ptr(g), B, S, C.byref(loss)),
                    "forward_backward")
        return float(loss.value)

    def adamw(self, opt: AdamW, step: int):
        o = _AdamWCfg(opt.lr, opt.beta1, opt.beta2, opt.eps, opt.weight_decay)
        self._check(lib().llmcu_adamw(self._h, C.byref(o), step), "adamw")

    def train_step(self, tokens: np.ndarray, targets: np.ndarray, opt: AdamW, step: int) -> float:
        t, g = self._batch(tokens, targets)
        B, S = t.shape
        o = _AdamWCfg(opt.lr, opt.beta1, opt.beta2, opt.eps, opt.weight_decay)
        loss = C.c_float()
        self._check(lib().llmcu_train_step(self._h, _ptr(t), _ptr(g), B, S, C.byref(o), step, C.byref(loss)),
                    "train_step")
        return float(loss.value)

    def train_step_device(self, d_tokens: int, d_targets: int, batch: int, seq: int, opt: AdamW, step: int):
        o = _AdamWCfg(opt.lr, opt.beta1, opt.beta2, opt.eps, opt.weight_decay)
        self._check(lib().llmcu_train_step_device(self._h, C.c_void_p(d_tokens), C.c_void_p(d_targets), batch,
                                                  seq, C.byref(o), step), "train_step_device")

    def read_loss(self) -> float:
        loss = C.c_float()
        self._check(lib().llmcu_read_loss(self._h, C.byref(loss)), "read_loss")
        return float(loss.value)

    # -- files
    def save_lora(self, directory: str, step: int):
        self._check(lib().llmcu_save_lora(self._h, directory.encode(), step), "save_lora")

    def load_lora(self, directory: str, step: int):
        self._check(lib().llmcu_load_lora(self._h, directory.encode(), step), "load_lora")

    def generate(self, prompt, n_new: int, want_logits: bool = False):
        """Greedy continuation of one prompt: (tokens [n], logits [n_new, V] or None,
        decode ms per token).  n excludes Qwen3's end ids and what follows."""
        p = np.ascontiguousarray(np.asarray(prompt, dtype=np.int32).reshape(-1))
        toks = np.zeros(n_new, dtype=np.int32)
        n_out = C.c_int(0)
        ms = C.c_float(0.0)
        logits = np.zeros((n_new, self.model.vocab), dtype=np.float32) if want_logits else None
        self._check(lib().llmcu_generate(self._h, _ptr(p), p.size, n_new, _ptr(toks), C.byref(n_out),
                                         _ptr(logits) if want_logits else None, C.byref(ms)), "generate")
        return toks[: n_out.value], logits, float(ms.value)

    def save_adamw_state(self, directory: str, step: int):
        """AdamW moments of every adapter to directory/lora_step{step}_adamw.bin."""
        self._check(lib().llmcu_save_adamw_state(self._h, directory.encode(), step), "save_adamw_state")

    def load_adamw_state(self, directory: str, step: int):
        self._check(lib().llmcu_load_adamw_state(self._h, directory.encode(), step), "load_adamw_state")

    # -- profiling
    def profile_enable(self, on: bool = True):
        self._check(lib().llmcu_profile_enable(self._h, int(on)), "profile_enable")

    def profile_read(self, reset: bool = True) -> dict:
        import json
        buf = C.create_string_buffer(4096)
        self._check(lib().llmcu_profile_read(self._h, buf, 4096, int(reset)), "profile_read")
        return json.loads(buf.value.decode())

    # -- data parallel
    @staticmethod
    def dp_unique_id() -> bytes:
        buf = (C.c_ubyte * 128)()
        st = lib().llmcu_dp_get_unique_id(buf)
        if st != OK:
            raise LlmcuError(st, "dp_get_unique_id")
        return bytes(buf)

    def dp_init(self, uid: bytes, rank: int, world: int):
        buf = (C.c_ubyte * 128).from_buffer_copy(uid)
        self._check(lib().llmcu_dp_init(self._h, buf, rank, world), "dp_init")

    def dp_set_timeout_ms(self, ms: int):
        self._check(lib().llmcu_dp_set_timeout_ms(self._h, ms), "dp_set_timeout_ms")


# ---------------------------------------------------------------- kernels
def _chk(st, what):
    if st != OK:
        raise LlmcuError(st, what)


def gemm_nt_f16(A_ptr, B_ptr, C_ptr, M, N, K, lda, ldb, ldc, stream=0):
    _chk(lib().llmcu_gemm_nt_f16(A_ptr, B_ptr, C_ptr, M, N, K, lda, ldb, ldc, stream), "gemm_nt_f16")


def gemm_nn_f16(A_ptr, B_ptr, C_ptr, M, N, K, lda, ldb, ldc, stream=0):
    _chk(lib().llmcu_gemm_nn_f16(A_ptr, B_ptr, C_ptr, M, N, K, lda, ldb, ldc, stream), "gemm_nn_f16")


def attention_fwd(q, k, v, o, lse, batch, seq, nh, nkv, hd, ldq, ldk, ldv, stream=0):
    _chk(lib().llmcu_attention_fwd(q, k, v, o, lse, batch, seq, nh, nkv, hd, ldq, ldk, ldv, stream),
         "attention_fwd")


def attention_bwd(q, k, v, o, do, lse, delta, dq, dk, dv, batch, seq, nh, nkv, hd, ldq, ldk, ldv, lddv,
                  stream=0):
    _chk(lib().llmcu_attention_bwd(q, k, v, o, do, lse, delta, dq, dk, dv, batch, seq, nh, nkv, hd, ldq, ldk,
                                   ldv, lddv, stream), "attention_bwd")


def attention_bwd_noalloc(q, k, v, o, do, lse, dq, dk, dv, batch, seq, nh, nkv, hd, ldq, ldk, ldv, lddv,
                          stream=0) -> int:
    """Allocation-free attention backward; returns the raw status (callers
    check LLMCU_ERR_UNSUPPORTED for sizes above the library's fixed scratch)."""
    return lib().llmcu_attention_bwd_noalloc(q, k, v, o, do, lse, dq, dk, dv, batch, seq, nh, nkv, hd, ldq,
                                             ldk, ldv, lddv, stream)


class LoraFiles:
    """The adapter files of one layout on the host alone (llmcu_lora_files_*):
    no device or context.  Adapters are given and returned as the golden's
    dict {"L{l}.{proj}.{A,B}": array} and laid out flat as the library keeps
    them (per layer, per target projection: A [r, d_in] then B [d_out, r])."""

    def __init__(self, model: Model, lora: Lora):
        self.model, self.lora = model, lora
        self._lay = _LoraLayout(model.n_layers, model.hidden, model.n_heads * model.head_dim,
                                model.n_kv_heads * model.head_dim, model.ffn, lora.rank, lora.targets)
        self.count = int(lib().llmcu_lora_layout_count(C.byref(self._lay)))
        if self.count <= 0:
            raise LlmcuError(1, "invalid adapter layout")

    def _dims(self, proj: int):
        m = self.model
        Q, KV = m.n_heads * m.head_dim, m.n_kv_heads * m.head_dim
        return {P_Q: (Q, m.hidden), P_K: (KV, m.hidden), P_V: (KV, m.hidden), P_O: (m.hidden, Q),
                P_GATE: (m.ffn, m.hidden), P_UP: (m.ffn, m.hidden), P_DOWN: (m.hidden, m.ffn)}[proj]

    def _slots(self):
        off = 0
        for l in range(self.model.n_layers):
            for p in self.lora.projs():
                d_out, d_in = self._dims(p)
                for mat, shape in (("A", (self.lora.rank, d_in)), ("B", (d_out, self.lora.rank))):
                    n = shape[0] * shape[1]
                    yield f"L{l}.{PROJ_NAMES[p]}.{mat}", off, shape
                    off += n

    def flatten(self, adapters: dict) -> np.ndarray:
        flat = np.empty(self.count, np.float32)
        for key, off, shape in self._slots():
            flat[off:off + shape[0] * shape[1]] = np.asarray(adapters[key], np.float32).reshape(-1)
        return flat

    def unflatten(self, flat: np.ndarray) -> dict:
        return {key: flat[off:off + shape[0] * shape[1]].reshape(shape).copy() for key, off, shape in self._slots()}

    def write(self, adapters: dict, directory: str, step: int):
        flat = self.flatten(adapters)
        _chk(lib().llmcu_lora_files_write(C.byref(self._lay), _ptr(flat), directory.encode(), step),
             f"lora_files_write {directory}")

    def read(self, directory: str, step: int) -> dict:
        flat = np.empty(self.count, np.float32)
        _chk(lib().llmcu_lora_files_read(C.byref(self._lay), _ptr(flat), directory.encode(), step),
             f"lora_files_read {directory}")
        return self.unflatten(flat)


def kernel_checks(stream=0) -> int:
    """Synchronises `stream`, then reads and clears the current device's error
    word of the kernel-level entry points; raises LlmcuError (DEVICE_CHECK)
    if any of their kernels gave up a bounded wait, else returns 0."""
    bits = C.c_int(0)
    st = lib().llmcu_kernel_checks(stream, C.byref(bits))
    if st != OK:
        raise LlmcuError(st, f"kernel-level device checks failed (error bits 0x{bits.value:x})")
    return bits.value


def kernel_wait_selftest(stream=0):
    """Launches the bounded-wait self-test (one wait that nothing satisfies;
    it gives up after 4 s); kernel_checks afterwards raises DEVICE_CHECK."""
    _chk(lib().llmcu_kernel_wait_selftest(stream), "kernel_wait_selftest")


def quantize_int8_rows(w_ptr, rows, cols, q_ptr, scale_ptr, stream=0):
    _chk(lib().llmcu_quantize_int8_rows(w_ptr, rows, cols, q_ptr, scale_ptr, stream), "quantize_int8_rows")
