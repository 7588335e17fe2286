"""The adapter files against the reference's own tooling (CPU, no GPU).

llm.cu's python/save_lora.py reads the trainer's adapter files
(weights/lora_step{N}_layer{l}_{wq,wk,wv,wo}_{A,B}.bin, raw fp32, A [16, d_in],
B [d_out, 16], src/train.cu:146-170) with the Qwen3-1.7B dimensions hard-coded
(save_lora.py:21-57) and converts them to and from a PEFT state dict
(save_lora.py:81-113).  Here the library's host-side writer and reader
(llmcu_lora_files_write / _read -- the file half of llmcu_save_lora /
llmcu_load_lora, whose device half tests/test_gpu_files.py checks on
the GPU) meet the UNMODIFIED save_lora.py, run from the reference checkout
beside this repository:

  library files --(save_lora.py --to-hf)--> PEFT tensors == the adapters set
  PEFT adapter --(save_lora.py --from-hf)--> files --(library reader)--> == the PEFT tensors

The test is skipped where the reference checkout is absent."""
import os
import subprocess
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REFERENCE = os.environ.get("LLMCU_REFERENCE_DIR", os.path.join(os.path.dirname(ROOT), "reference"))
SAVE_LORA = os.path.join(REFERENCE, "python", "save_lora.py")
HF = {"wq": "self_attn.q_proj", "wk": "self_attn.k_proj", "wv": "self_attn.v_proj", "wo": "self_attn.o_proj"}


def _peft_key(layer, proj, mat):
    return f"base_model.model.model.layers.{layer}.{HF[proj]}.lora_{mat}.weight"


@pytest.fixture(scope="module")
def files_1p7b(llmcu):
    from oracle import golden as G
    cfg = G.CFG_QWEN3_1P7B
    model = llmcu.Model.qwen3_1p7b()
    return cfg, llmcu.LoraFiles(model, llmcu.Lora(cfg.lora_rank, cfg.lora_alpha))


def test_layout_count_and_invalid_layouts(llmcu, files_1p7b):
    cfg, lf = files_1p7b
    assert lf.count == cfg.n_lora_params() == 6_422_528
    with pytest.raises(llmcu.LlmcuError):
        llmcu.LoraFiles(llmcu.Model.qwen3_1p7b(), llmcu.Lora(17, 32.0))


def test_missing_and_short_files_are_io_errors(llmcu, tmp_path):
    from oracle import golden as G
    cfg = G.CFG_TINY
    lf = llmcu.LoraFiles(llmcu.Model.tiny(), llmcu.Lora(cfg.lora_rank, cfg.lora_alpha))
    lora = G.make_lora(cfg, 3)
    lf.write(lora, str(tmp_path), 2)
    got = lf.read(str(tmp_path), 2)
    assert all(np.array_equal(got[k], lora[k]) for k in lora)
    with pytest.raises(llmcu.LlmcuError) as e:
        lf.read(str(tmp_path), 3)
    assert e.value.status == 4
    p = tmp_path / "lora_step2_layer1_wo_B.bin"
    p.write_bytes(p.read_bytes()[:-4])
    with pytest.raises(llmcu.LlmcuError) as e:
        lf.read(str(tmp_path), 2)
    assert e.value.status == 4


@pytest.mark.skipif(not os.path.exists(SAVE_LORA), reason="reference checkout (python/save_lora.py) not present")
def test_reference_save_lora_reads_and_writes_the_library_files(llmcu, files_1p7b, tmp_path):
    import torch
    from oracle import golden as G
    cfg, lf = files_1p7b
    lora = G.make_lora(cfg, 77)
    wdir = tmp_path / "weights"
    wdir.mkdir()
    lf.write(lora, str(wdir), 100)
    names = sorted(os.listdir(wdir))
    assert len(names) == cfg.n_layers * 4 * 2 and all(n.startswith("lora_step100_layer") for n in names)

    listing = subprocess.run([sys.executable, SAVE_LORA, "--list", "--step", "100", "--weights-dir", str(wdir)],
                             capture_output=True, text=True, check=True, timeout=600).stdout
    assert "MISSING" not in listing and "6,422,528" in listing

    out = tmp_path / "peft_step100.pt"
    subprocess.run([sys.executable, SAVE_LORA, "--to-hf", "--step", "100", "--out", str(out), "--weights-dir",
                    str(wdir)], capture_output=True, text=True, check=True, timeout=600)
    state = torch.load(str(out), map_location="cpu")
    assert len(state) == cfg.n_layers * 4 * 2
    for l in range(cfg.n_layers):
        for p in HF:
            for mat in ("A", "B"):
                t = state[_peft_key(l, p, mat)].numpy()
                assert t.dtype == np.float32 and np.array_equal(t, lora[f"L{l}.{p}.{mat}"]), (l, p, mat)

    # a PEFT adapter the other way: save_lora.py --from-hf writes the files, the library reads them
    other = G.make_lora(cfg, 78)
    peft = {_peft_key(l, p, mat): torch.from_numpy(other[f"L{l}.{p}.{mat}"])
            for l in range(cfg.n_layers) for p in HF for mat in ("A", "B")}
    adapter = tmp_path / "adapter.pt"
    torch.save(peft, str(adapter))
    back = tmp_path / "from_hf"
    subprocess.run([sys.executable, SAVE_LORA, "--from-hf", "--adapter", str(adapter), "--step", "0",
                    "--weights-dir", str(back)], capture_output=True, text=True, check=True, timeout=600)
    got = lf.read(str(back), 0)
    assert set(got) == set(other)
    assert all(np.array_equal(got[k], other[k]) for k in other)
