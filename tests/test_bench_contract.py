"""bench.py's host-side pieces, on CPU: the algorithmic work it divides by
(the step's FLOPs per token at the Qwen3-1.7B shape), the token windows of
its workloads, the adapter-target parsing and the parsing of the
nvidia-smi clock samples that decide whether a run is kept."""
import importlib.util
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def bench():
    spec = importlib.util.spec_from_file_location("bench_under_test", os.path.join(ROOT, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


@pytest.fixture(scope="module")
def model():
    sys.path.insert(0, os.path.join(ROOT, "llm.cu_b200"))
    import llmcu
    return llmcu.Model.qwen3_1p7b()


def test_flops_per_token_at_the_c2_shape(bench, model):
    # frozen linears per layer: q, k, v, o, gate, up, down (out x in)
    per_layer = 2048 * 2048 + 2 * 1024 * 2048 + 2048 * 2048 + 3 * 6144 * 2048
    n_lin = 28 * per_layer + 151936 * 2048  # + the tied lm_head
    assert n_lin == 1_720_451_072
    assert bench.algorithmic_gemm_flops_per_token(model) == 4 * n_lin
    assert bench.layer_gemm_flops_per_token(model) + bench.lm_head_flops_per_token(model) == 4 * n_lin
    # rank-16 adapters on q, k, v, o: r (in + out) parameters each
    n_lora = 28 * 16 * ((2048 + 2048) + 2 * (2048 + 1024) + (2048 + 2048))
    assert n_lora == 6_422_528
    attn = 3 * 2 * 512 * 128 * 16 * 28  # causal forward + backward at seq 512
    total = bench.algorithmic_flops_per_token(model, 512, n_lora)
    assert total == 4 * n_lin + attn + 6 * n_lora
    assert abs(total / 1e9 - 7.097) < 1e-3


def test_token_windows(bench):
    tok, tgt = bench.make_tokens(151936, 8, 512, 1000, "zipf")
    assert tok.shape == (8, 512) and tgt.shape == (8, 512)
    assert tok.dtype == np.int32 and tok.flags["C_CONTIGUOUS"] and tgt.flags["C_CONTIGUOUS"]
    assert np.array_equal(tok[:, 1:], tgt[:, :-1])  # targets are the next token
    assert tok.min() >= 0 and max(tok.max(), tgt.max()) < 151936
    # Zipf(1.1): the first id is the most frequent one
    counts = np.bincount(tok.ravel(), minlength=4)
    assert counts[0] == counts.max()
    tok2, _ = bench.make_tokens(151936, 8, 512, 1000, "zipf")
    assert np.array_equal(tok, tok2)
    tok3, _ = bench.make_tokens(151936, 8, 512, bench.shard_seed(1), "zipf")
    assert not np.array_equal(tok, tok3)  # each rank draws its own sequences
    tu, _ = bench.make_tokens(4096, 2, 32, 7, "uniform")
    assert tu.min() >= 0 and tu.max() < 4096


def test_lora_targets(bench):
    assert bench.parse_targets("attn") == ("wq", "wk", "wv", "wo")
    assert bench.parse_targets("mlp") == ("w_gate", "w_up", "w_down")
    assert len(bench.parse_targets("all")) == 7
    assert bench.parse_targets("w_down, wq") == ("wq", "w_down")  # canonical order
    with pytest.raises(SystemExit):
        bench.parse_targets("wq,w_nope")
    with pytest.raises(SystemExit):
        bench.parse_targets(",")


def test_clock_samples(bench):
    rows = [
        "0, 1590, 1965, 612.40, 0x0000000000000004, Not Active, Not Active, Not Active, Active\n",
        "0, 1605, 1965, 871.10, 0x0000000000000004, Not Active, Not Active, Not Active, Active\n",
        "0, 1575, 1965, [N/A], 0x0000000000000000, Not Active, Not Active, Not Active, Not Active\n",
        "garbage line\n",
    ]
    c = bench.ClockSampler.summarise(rows)
    assert c["sm_mhz"] == 1590.0 and c["sm_max_mhz"] == 1965.0
    assert c["reasons"] == ["sw_power_cap"] and c["samples"] == 3
    assert c["power_w_max"] == 871.1
    hot = bench.ClockSampler.summarise(
        ["0, 1200, 1965, 700, 0x48, Not Active, Active, Not Active, Active\n"])
    assert hot["reasons"] == ["hw_thermal_slowdown", "sw_power_cap"]  # a run the driver rejects
    assert bench.ClockSampler.summarise([]) is None
    assert bench.ClockSampler.summarise(["0, [N/A], [N/A], [N/A], x, a, b, c, d\n"])["power_w_max"] is None
