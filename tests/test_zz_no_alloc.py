"""GPU test of llmcu_attention_bwd_noalloc, the attention backward entry point
that allocates nothing: it keeps its row sums in a fixed array inside the
library instead of a caller-provided scratch buffer, for callers that cannot
call cudaMalloc (a caching allocator owns the device memory, or a
latency-critical loop cannot afford cudaMalloc's implicit synchronisation).

The noalloc and scratch-buffer entry points run the same kernels on the same
inputs, so dK and dV (accumulated inside one CTA in a fixed order) must be
bit-identical and dQ (reduce-added by the key tiles in no fixed order) equal
to fp32 rounding; this holds on two calls in a row with different shapes, so
a stale array from the first call cannot leak into the second.  The first
shape is also checked directly against an fp32 torch autograd reference at
the attention tolerance used elsewhere (rel-L2 1e-2).  A row stride the TMA
descriptors refuse is UNSUPPORTED, as for the scratch-buffer entry point, and
the device checks report no wait that gave up.  The file name makes pytest
collect it last."""
import math

import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

UNSUPPORTED = 8


def rel_l2(a, b):
    a = a.double().flatten()
    b = b.double().flatten()
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


def _torch_ref(q, k, v, do, B, S, nh, nkv, hd):
    """fp32 autograd gradients of causal GQA attention (scale 1/sqrt(hd))."""
    qf, kf, vf = (t.float().requires_grad_(True) for t in (q, k, v))
    qh = qf.view(B, S, nh, hd).transpose(1, 2)
    kh = kf.view(B, S, nkv, hd).repeat_interleave(nh // nkv, dim=2).transpose(1, 2)
    vh = vf.view(B, S, nkv, hd).repeat_interleave(nh // nkv, dim=2).transpose(1, 2)
    s = (qh @ kh.transpose(-1, -2)) / math.sqrt(hd)
    s = s.masked_fill(torch.ones(S, S, dtype=torch.bool, device=q.device).triu(1), float("-inf"))
    o = (torch.softmax(s, dim=-1) @ vh).transpose(1, 2).reshape(B * S, nh * hd)
    o.backward(do.float())
    return qf.grad, kf.grad, vf.grad


def _case(llmcu, dev, B, S, nh, nkv, hd, seed, against_torch=False):
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
        assert llmcu.kernel_checks(st) == 0  # synchronises; no bounded wait gave up
        outs[name] = (dq, dk, dv)
    (dq_n, dk_n, dv_n), (dq_r, dk_r, dv_r) = outs["noalloc"], outs["ref"]
    assert torch.isfinite(dq_n).all() and torch.isfinite(dk_n).all() and torch.isfinite(dv_n.float()).all()
    assert torch.equal(dk_n, dk_r)
    assert torch.equal(dv_n, dv_r)
    assert rel_l2(dq_n, dq_r) <= 1e-5
    if against_torch:
        gq, gk, gv = _torch_ref(q, k, v, do, B, S, nh, nkv, hd)
        assert rel_l2(dq_n, gq) < 1e-2
        assert rel_l2(dk_n, gk) < 1e-2
        assert rel_l2(dv_n.float(), gv) < 1e-2


def test_noalloc_matches_scratch_entry_on_two_calls(llmcu, cuda_device):
    # first call: the larger problem fills more of the library's array
    _case(llmcu, cuda_device, 4, 384, 16, 8, 128, seed=1, against_torch=True)
    # second call: a smaller, ragged problem reading only its own fresh sums
    _case(llmcu, cuda_device, 1, 200, 4, 2, 64, seed=2)


def test_noalloc_rejects_sizes_beyond_its_array_and_unaligned_strides(llmcu, cuda_device):
    dev = cuda_device
    st = torch.cuda.current_stream().cuda_stream
    buf = torch.zeros(1024, device=dev, dtype=torch.float32)
    p = buf.data_ptr()
    # 2 x 16 heads x 32769 tokens = 1,048,608 rows of sums > 1,048,576: refused before any launch
    status = llmcu.attention_bwd_noalloc(p, p, p, p, p, p, p, p, p, 2, 32769, 16, 8, 128, 2048, 1024, 1024, 1024, st)
    assert status == UNSUPPORTED
    # a q row stride of 2052 halves (4104 bytes, not a multiple of 16) is refused by the TMA
    # descriptor before the attention kernel launches, as it is for llmcu_attention_bwd
    B, S, nh, nkv, hd = 1, 64, 16, 8, 128
    M = B * S
    q = torch.zeros(M, nh * hd + 4, device=dev, dtype=torch.float16)
    kv = torch.zeros(M, nkv * hd, device=dev, dtype=torch.float16)
    o = torch.zeros(M, nh * hd, device=dev, dtype=torch.float16)
    lse = torch.zeros(B, nh, S, device=dev, dtype=torch.float32)
    dq = torch.zeros(M, nh * hd, device=dev, dtype=torch.float32)
    dk = torch.zeros(M, nkv * hd, device=dev, dtype=torch.float32)
    dv = torch.zeros(M, nkv * hd, device=dev, dtype=torch.float16)
    status = llmcu.attention_bwd_noalloc(q.data_ptr(), kv.data_ptr(), kv.data_ptr(), o.data_ptr(), o.data_ptr(),
                                         lse.data_ptr(), dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), B, S, nh, nkv,
                                         hd, nh * hd + 4, nkv * hd, nkv * hd, nkv * hd, st)
    assert status == UNSUPPORTED
    assert llmcu.kernel_checks(st) == 0
