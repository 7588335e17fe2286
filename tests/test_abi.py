"""CPU tests of the drop-in boundary: libllmcu.so loads, exports every entry
point include/llmcu.h declares, validates arguments without a GPU, and the
llm_train driver keeps the reference CLI.  No kernel is launched here."""
import ctypes as C
import os
import re
import subprocess

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "llmcu.h")


def declared_symbols():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(llmcu_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_the_boundary():
    syms = declared_symbols()
    for s in ("llmcu_ctx_create", "llmcu_train_step", "llmcu_forward_backward", "llmcu_get_lora_grads",
              "llmcu_adamw", "llmcu_save_lora", "llmcu_quantize_int8_rows", "llmcu_dp_init",
              "llmcu_dp_set_timeout_ms", "llmcu_last_error", "llmcu_set_base_tensor", "llmcu_set_lora"):
        assert s in syms


def test_library_exports_every_declared_symbol(llmcu):
    lib = llmcu.lib()
    missing = [s for s in declared_symbols() if not hasattr(lib, s)]
    assert not missing, missing
    # the binding declares signatures for all of them
    assert set(declared_symbols()) <= set(llmcu.exported_symbols())


def test_version_and_null_handling(llmcu):
    lib = llmcu.lib()
    assert lib.llmcu_version().decode().startswith("llmcu")
    assert lib.llmcu_last_error(None) == b"null context"
    assert lib.llmcu_device_bytes(None) == 0
    assert lib.llmcu_ctx_create(None, None, None, 0, None) == 1          # INVALID_ARG
    assert lib.llmcu_quantize_int8_rows(None, 4, 4, None, None, None) == 1
    assert lib.llmcu_dp_get_unique_id(None) == 1
    assert lib.llmcu_synchronize(None) == 1


def test_ctx_create_rejects_unsupported_configs(llmcu):
    """Config validation happens before any device call."""
    cases = [
        (llmcu.Model(256, 2, 4, 2, 96, 768, 4096), llmcu.Lora(4, 8.0), llmcu.Run(1, 32), 8),   # head_dim 96
        (llmcu.Model(256, 2, 4, 3, 64, 768, 4096), llmcu.Lora(4, 8.0), llmcu.Run(1, 32), 1),   # 4 % 3 heads
        (llmcu.Model(256, 2, 4, 2, 64, 768, 4096), llmcu.Lora(32, 8.0), llmcu.Run(1, 32), 8),  # rank 32
        (llmcu.Model(256, 2, 4, 2, 64, 700, 4096), llmcu.Lora(4, 8.0), llmcu.Run(1, 32), 8),   # ffn % 128
        (llmcu.Model(256, 2, 4, 2, 64, 768, 4096), llmcu.Lora(4, 8.0), llmcu.Run(0, 32), 1),   # batch 0
        (llmcu.Model(256, 2, 4, 2, 64, 768, 4096), llmcu.Lora(4, 8.0, 0x80), llmcu.Run(1, 32), 1),  # target bit 7
        # MLP targets put their side columns on 256-column tile boundaries
        (llmcu.Model(256, 2, 4, 2, 64, 640, 4096), llmcu.Lora(4, 8.0, llmcu.TARGETS_ALL), llmcu.Run(1, 32), 8),
    ]
    for model, lora, run, want in cases:
        with pytest.raises(llmcu.LlmcuError) as ei:
            llmcu.Context(model, lora, run)
        assert ei.value.status == want


def test_ctx_create_without_a_gpu_reports_cuda_error(llmcu):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    with pytest.raises(llmcu.LlmcuError) as ei:
        llmcu.Context(llmcu.Model.tiny(), llmcu.Lora(4, 8.0), llmcu.Run(1, 32))
    assert ei.value.status == 2


def test_llm_train_keeps_the_reference_cli():
    exe = os.path.join(ROOT, "llm.cu_b200", "llm_train")
    if not os.path.exists(exe):
        pytest.skip("llm_train not built")
    out = subprocess.run([exe, "--help"], capture_output=True, text=True, timeout=30).stdout
    for flag in ("--lr", "--steps", "--seq-len", "--save-every", "--log-every"):
        assert flag in out
    # missing data file -> the reference's error text and exit status 1 (src/train.cu:195-200)
    r = subprocess.run([exe, "--data", "/nonexistent/train_tokens.bin", "--config", "tiny"], capture_output=True,
                       text=True, timeout=30)
    assert r.returncode == 1 and "not found" in r.stderr


def test_ref_io_round_trip(tmp_path):
    import sys
    sys.path.insert(0, os.path.join(ROOT, "tests", "golden"))
    import ref_io
    from oracle import golden as G
    cfg = G.CFG_TINY
    base = G.make_base_weights(cfg, 1)
    lora = G.make_lora(cfg, 2)
    tok, tgt = G.make_tokens(cfg, 2, 8, 3)
    p = tmp_path / "in.bin"
    ref_io.write_input(str(p), cfg, base, lora, tok, tgt)
    n_w = sum(v.size for v in base.values())
    n_l = sum(v.size for v in lora.values())
    assert p.stat().st_size == 4 * (10 + 2 * tok.size + 5 + n_w + n_l)
    # an output file with known content parses back into the same dict layout
    out = tmp_path / "out.bin"
    vals = np.arange(2 + 2 * n_l, dtype=np.float32)
    vals.tofile(out)
    losses, grads, after = ref_io.read_output(str(out), cfg, 2)
    assert losses.tolist() == [0.0, 1.0]
    assert grads["L0.wq.A"].shape == (4, 256) and after["L1.wo.B"].shape == (256, 4)
    assert grads["L0.wq.A"].ravel()[0] == 2.0


def test_config_structs_match_the_header(llmcu, tmp_path):
    """The ctypes mirrors of the config structs have the C layout: every
    field at the offset (and the struct at the size) a C compiler gives the
    header's definition."""
    structs = {"llmcu_model_cfg": llmcu._ModelCfg, "llmcu_lora_cfg": llmcu._LoraCfg,
               "llmcu_run_cfg": llmcu._RunCfg, "llmcu_adamw_cfg": llmcu._AdamWCfg}
    lines = ['#include <stddef.h>', '#include <stdio.h>', '#include "llmcu.h"', "int main(void) {"]
    for cname, py in structs.items():
        lines.append(f'  printf("{cname} size %zu\\n", sizeof({cname}));')
        for fname, _ in py._fields_:
            lines.append(f'  printf("{cname} {fname} %zu\\n", offsetof({cname}, {fname}));')
    lines += ["  return 0;", "}"]
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines) + "\n")
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-std=c99", "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe)], check=True,
                   timeout=60)
    out = subprocess.run([str(exe)], capture_output=True, text=True, check=True, timeout=30).stdout.split("\n")
    got = {tuple(l.split()[:2]): int(l.split()[2]) for l in out if l.strip()}
    for cname, py in structs.items():
        assert got[(cname, "size")] == C.sizeof(py), cname
        for fname, _ in py._fields_:
            assert got[(cname, fname)] == getattr(py, fname).offset, (cname, fname)


def test_llm_train_rejects_unknown_lora_targets():
    exe = os.path.join(ROOT, "llm.cu_b200", "llm_train")
    if not os.path.exists(exe):
        pytest.skip("llm_train not built")
    r = subprocess.run([exe, "--config", "tiny", "--synthetic", "--lora-targets", "wq,w_bogus"], capture_output=True,
                       text=True, timeout=30)
    assert r.returncode == 1
    assert "unknown --lora-targets entry 'w_bogus'" in r.stderr


def test_step_inputs_must_share_one_shape(llmcu):
    """The library copies batch * seq ids from each host pointer, so the
    binding refuses tokens and targets of different shapes before any call."""
    Ctx = llmcu.Context
    t, g = Ctx._batch(np.arange(6, dtype=np.int64).reshape(2, 3), [[1, 2, 3], [4, 5, 6]])
    assert t.dtype == np.int32 and g.dtype == np.int32 and t.flags.c_contiguous and t.shape == g.shape == (2, 3)
    for tok, tgt in [(np.zeros((2, 3)), np.zeros((2, 2))), (np.zeros((2, 3)), np.zeros((3, 2))),
                     (np.zeros(6), np.zeros(6)), (np.zeros((2, 3)), np.zeros((1, 3)))]:
        with pytest.raises(ValueError):
            Ctx._batch(tok, tgt)
