"""GPU test of llmcu_attention_bwd_noalloc, the attention backward entry point
that allocates nothing: it keeps its row sums in a fixed array inside the
library instead of a caller-provided scratch buffer, for callers that cannot
call cudaMalloc (a caching allocator owns the device memory, or a
latency-critical loop cannot afford cudaMalloc's implicit synchronisation).

Its results must equal those of llmcu_attention_bwd (which takes the scratch
from the caller) within the attention tolerance used elsewhere (rel-L2 1e-2),
on two calls in a row with different shapes, so that a stale array from the
first call cannot leak into the second.  The file name makes pytest collect it
last."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

UNSUPPORTED = 8


def rel_l2(a, b):
    a = a.double().flatten()
    b = b.double().flatten()
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


def _case(llmcu, dev, B, S, nh, nkv, hd, seed):
    g = torch.Generator(device="cpu").manual_seed(seed)
    M = B * S
    q = torch.randn(M, nh * hd, generator=g).half().to(dev)
    k = torch.randn(M, nkv * hd, generator=g).half().to(dev)
    v = torch.randn(M, nkv * hd, generator=g).half().to(dev)
    do = torch.randn(M, nh * hd, generator=g).half().to(dev)
    o = torch.empty(M, nh * hd, device=dev, dtype=torch.float16)
    lse = torch.empty(B, nh, S, device=dev, dtype=torch.float32)
    st = torch.cuda.current_stream().cuda_stream
    llmcu.attention_fwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), lse.data_ptr(), B, S, nh, nkv, hd,
                        nh * hd, nkv * hd, nkv * hd, st)
    outs = {}
    for name in ("ref", "noalloc"):
        dq = torch.full((M, nh * hd), float("nan"), device=dev, dtype=torch.float32)
        dk = torch.full((M, nkv * hd), float("nan"), device=dev, dtype=torch.float32)
        dv = torch.full((M, nkv * hd), float("nan"), device=dev, dtype=torch.float16)
        if name == "ref":
            delta = torch.empty(B, nh, S, device=dev, dtype=torch.float32)
            llmcu.attention_bwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), do.data_ptr(), lse.data_ptr(),
                                delta.data_ptr(), dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), B, S, nh, nkv, hd,
                                nh * hd, nkv * hd, nkv * hd, nkv * hd, st)
        else:
            status = llmcu.attention_bwd_noalloc(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), do.data_ptr(),
                                                 lse.data_ptr(), dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), B, S, nh,
                                                 nkv, hd, nh * hd, nkv * hd, nkv * hd, nkv * hd, st)
            assert status == 0
        torch.cuda.synchronize()
        outs[name] = (dq, dk, dv)
    for a, b in zip(outs["noalloc"], outs["ref"]):
        assert torch.isfinite(a.float()).all()
        assert rel_l2(a.float(), b.float()) <= 1e-2


def test_noalloc_matches_scratch_entry_on_two_calls(llmcu, cuda_device):
    # first call: the larger problem fills more of the library's array
    _case(llmcu, cuda_device, 4, 384, 16, 8, 128, seed=1)
    # second call: a smaller, ragged problem reading only its own fresh sums
    _case(llmcu, cuda_device, 1, 200, 4, 2, 64, seed=2)


def test_noalloc_rejects_sizes_beyond_its_array(llmcu, cuda_device):
    dev = cuda_device
    buf = torch.zeros(1024, device=dev, dtype=torch.float32)
    p = buf.data_ptr()
    # 2 x 16 heads x 32769 tokens = 1,048,608 rows of sums > 1,048,576: refused before any launch
    status = llmcu.attention_bwd_noalloc(p, p, p, p, p, p, p, p, p, 2, 32769, 16, 8, 128, 2048, 1024, 1024, 1024,
                                         torch.cuda.current_stream().cuda_stream)
    assert status == UNSUPPORTED
