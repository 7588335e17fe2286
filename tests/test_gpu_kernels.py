"""Kernel-level parity on the GPU: each CUDA kernel, called through the C ABI
(libllmcu.so), against a plain PyTorch fp32 reference of the same op on the
same fp16 inputs.

Tolerances: GEMM outputs to 1e-3 relative L2 (fp32 accumulation of exact fp16
products; only summation order differs).  Attention to 1e-2 relative L2
(probabilities are rounded to fp16 before the P.V and dS.K products)."""
import math
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


def rel_l2(a, b):
    a = a.detach().double().flatten()
    b = b.detach().double().flatten()
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


# (4096, 2048, *) leave a partial last wave that runs split along K (the
# tail split); every shape runs twice to check the split's counters re-arm.
@pytest.mark.parametrize("M,N,K", [(4096, 4096, 2048), (32, 64, 256), (200, 300, 200), (128, 151936 // 8, 2048),
                                   (1000, 2048, 6144), (4096, 2048, 2048), (4096, 2048, 12288), (640, 12288, 2048),
                                   # one row; the shortest K a 16-byte row stride allows
                                   (1, 256, 64), (129, 520, 8)])
def test_gemm_nt_matches_torch(llmcu, cuda_device, M, N, K):
    g = torch.Generator(device="cpu").manual_seed(M * 7 + N)
    A = torch.randn(M, K, generator=g).half().to(cuda_device)
    B = torch.randn(N, K, generator=g).half().to(cuda_device)
    ref = A.float() @ B.float().t()
    for _ in range(2):
        C = torch.full((M, N), float("nan"), device=cuda_device, dtype=torch.float32)
        llmcu.gemm_nt_f16(A.data_ptr(), B.data_ptr(), C.data_ptr(), M, N, K, K, K, N,
                          torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        assert torch.isfinite(C).all()
        assert rel_l2(C, ref) < 1e-3


@pytest.mark.parametrize("M,N,K", [(4096, 2048, 2048), (32, 64, 256), (200, 296, 200), (4096, 6144, 2048),
                                   (1000, 2112, 4096), (1, 64, 64), (130, 8, 72)])
def test_gemm_nn_matches_torch(llmcu, cuda_device, M, N, K):
    """B read MN-major ([K, N] row-major), the input-gradient GEMMs' operand.
    Row strides must be multiples of 16 bytes (TMA), so N is a multiple of 8."""
    g = torch.Generator(device="cpu").manual_seed(M * 5 + N)
    A = torch.randn(M, K, generator=g).half().to(cuda_device)
    B = torch.randn(K, N, generator=g).half().to(cuda_device)
    ref = A.float() @ B.float()
    C = torch.full((M, N), float("nan"), device=cuda_device, dtype=torch.float32)
    llmcu.gemm_nn_f16(A.data_ptr(), B.data_ptr(), C.data_ptr(), M, N, K, K, N, N,
                      torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert torch.isfinite(C).all()
    assert rel_l2(C, ref) < 1e-3


def _attn_ref(q, k, v, B, S, nh, nkv, hd):
    qh = q.view(B, S, nh, hd).transpose(1, 2)
    kh = k.view(B, S, nkv, hd).repeat_interleave(nh // nkv, dim=2).transpose(1, 2)
    vh = v.view(B, S, nkv, hd).repeat_interleave(nh // nkv, dim=2).transpose(1, 2)
    s = (qh @ kh.transpose(-1, -2)) / math.sqrt(hd)
    mask = torch.ones(S, S, dtype=torch.bool, device=q.device).triu(1)
    s = s.masked_fill(mask, float("-inf"))
    lse = torch.logsumexp(s, dim=-1)
    o = torch.softmax(s, dim=-1) @ vh
    return o.transpose(1, 2).reshape(B * S, nh * hd), lse


@pytest.mark.parametrize("B,S,nh,nkv,hd", [(2, 128, 4, 2, 64), (1, 32, 4, 2, 64), (2, 512, 16, 8, 128),
                                           (1, 200, 16, 8, 128), (1, 1000, 4, 2, 128),
                                           # ragged tiles in every sequence of a batch; a KV group of four
                                           (3, 333, 8, 4, 64), (2, 300, 8, 2, 128)])
def test_attention_fwd_bwd_matches_torch(llmcu, cuda_device, B, S, nh, nkv, hd):
    g = torch.Generator(device="cpu").manual_seed(S + nh)
    M = B * S
    q = torch.randn(M, nh * hd, generator=g).half().to(cuda_device)
    k = torch.randn(M, nkv * hd, generator=g).half().to(cuda_device)
    v = torch.randn(M, nkv * hd, generator=g).half().to(cuda_device)
    do = torch.randn(M, nh * hd, generator=g).half().to(cuda_device)
    o = torch.empty(M, nh * hd, device=cuda_device, dtype=torch.float16)
    lse = torch.empty(B, nh, S, device=cuda_device, dtype=torch.float32)
    st = torch.cuda.current_stream().cuda_stream
    llmcu.attention_fwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), lse.data_ptr(), B, S, nh, nkv,
                        hd, nh * hd, nkv * hd, nkv * hd, st)
    torch.cuda.synchronize()
    qf, kf, vf = (t.float().requires_grad_(True) for t in (q, k, v))
    o_ref, lse_ref = _attn_ref(qf, kf, vf, B, S, nh, nkv, hd)
    assert rel_l2(o.float(), o_ref) < 1e-2
    assert torch.allclose(lse, lse_ref, atol=2e-3, rtol=1e-4)

    o_ref.backward(do.float())
    delta = torch.empty(B, nh, S, device=cuda_device, dtype=torch.float32)
    dq = torch.empty(M, nh * hd, device=cuda_device, dtype=torch.float32)
    dk = torch.empty(M, nkv * hd, device=cuda_device, dtype=torch.float32)
    dv = torch.empty(M, nkv * hd, device=cuda_device, dtype=torch.float16)
    llmcu.attention_bwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), do.data_ptr(), lse.data_ptr(),
                        delta.data_ptr(), dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), B, S, nh, nkv, hd,
                        nh * hd, nkv * hd, nkv * hd, nkv * hd, st)
    torch.cuda.synchronize()
    assert rel_l2(dq, qf.grad) < 1e-2
    assert rel_l2(dk, kf.grad) < 1e-2
    assert rel_l2(dv.float(), vf.grad) < 1e-2


@pytest.mark.parametrize("rows,cols", [(64, 2048), (7, 13), (2048, 6144), (3, 1)])
def test_int8_quantiser_bit_exact(llmcu, cuda_device, rows, cols):
    from oracle.quant import quantize_rows
    rng = np.random.Generator(np.random.PCG64(rows * 1000 + cols))
    w = (rng.standard_normal((rows, cols), dtype=np.float32) * np.float32(0.02)).astype(np.float16).astype(np.float32)
    if rows >= 3:
        w[1] = 0.0                                     # all-zero row -> scale 0, q 0
        w[2, 0] = 0.5                                  # ties in w*inv around .5 are exercised by the draw
    q_ref, s_ref = quantize_rows(w)
    wd = torch.from_numpy(w).to(cuda_device)
    qd = torch.empty(rows, cols, dtype=torch.int8, device=cuda_device)
    sd = torch.empty(rows, dtype=torch.float32, device=cuda_device)
    llmcu.quantize_int8_rows(wd.data_ptr(), rows, cols, qd.data_ptr(), sd.data_ptr(),
                             torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert np.array_equal(qd.cpu().numpy(), q_ref)
    assert np.array_equal(sd.cpu().numpy().view(np.uint32), s_ref.view(np.uint32))


HARNESS = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle", "_ref",
                       "ref_harness_full")


@pytest.mark.skipif(not os.path.exists(HARNESS), reason="reference harness not built (make -C oracle/ref_harness)")
@pytest.mark.parametrize("rows,cols", [(64, 2048), (7, 13), (300, 6144)])
def test_int8_quantiser_matches_the_reference_kernel(llmcu, cuda_device, tmp_path, rows, cols):
    """The library's quantiser, the numpy restatement (oracle/quant.py) and the
    reference's own quantize_kernel (src/kernels/quantize.cu:8-50, run by the
    harness from the reference's sources) agree bit for bit on the same fp16
    draw: codes and scales, an all-zero row and exact .5 ties included."""
    import subprocess
    from oracle.quant import quantize_rows
    rng = np.random.Generator(np.random.PCG64(rows * 7 + cols))
    w = (rng.standard_normal((rows, cols), dtype=np.float32) * np.float32(0.02)).astype(np.float16).astype(np.float32)
    if rows >= 3:
        w[1] = 0.0
        w[2, :] = np.float32(0.25)
        w[2, 0] = np.float32(127.0 / 2.0)  # scale 0.5: every 0.25 is a tie at 0.5 (rounds to even 0)
    src = tmp_path / "w.bin"
    with open(src, "wb") as f:
        np.array([rows, cols], np.int32).tofile(f)
        w.tofile(f)
    out = tmp_path / "q.bin"
    subprocess.run([HARNESS, "quantize", str(src), str(out)], check=True, timeout=300)
    raw = np.fromfile(out, dtype=np.uint8)
    q_ref = raw[: rows * cols].view(np.int8).reshape(rows, cols)
    s_ref = raw[rows * cols:].view(np.float32)
    q_np, s_np = quantize_rows(w)
    wd = torch.from_numpy(w).to(cuda_device)
    qd = torch.empty(rows, cols, dtype=torch.int8, device=cuda_device)
    sd = torch.empty(rows, dtype=torch.float32, device=cuda_device)
    llmcu.quantize_int8_rows(wd.data_ptr(), rows, cols, qd.data_ptr(), sd.data_ptr(),
                             torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert np.array_equal(q_ref, q_np) and np.array_equal(s_ref.view(np.uint32), s_np.view(np.uint32))
    assert np.array_equal(qd.cpu().numpy(), q_ref)
    assert np.array_equal(sd.cpu().numpy().view(np.uint32), s_ref.view(np.uint32))


def test_bounded_wait_gives_up_and_is_reported(llmcu, cuda_device):
    """A wait that nothing satisfies ends after the kernels' bounded-wait limit
    with the error bit set; llmcu_kernel_checks reports it once and the device
    keeps working (a small attention forward afterwards is clean)."""
    import time
    st = torch.cuda.current_stream().cuda_stream
    assert llmcu.kernel_checks(st) == 0
    t0 = time.time()
    llmcu.kernel_wait_selftest(st)
    with pytest.raises(llmcu.LlmcuError) as e:
        llmcu.kernel_checks(st)
    elapsed = time.time() - t0
    assert e.value.status == 7  # LLMCU_ERR_DEVICE_CHECK
    assert "0x1" in str(e.value)
    assert 3.5 < elapsed < 60.0
    assert llmcu.kernel_checks(st) == 0  # read and cleared
    B, S, nh, nkv, hd = 1, 128, 2, 1, 128
    q = torch.randn(B * S, nh * hd, device=cuda_device).half()
    k = torch.randn(B * S, nkv * hd, device=cuda_device).half()
    v = torch.randn(B * S, nkv * hd, device=cuda_device).half()
    o = torch.empty(B * S, nh * hd, device=cuda_device, dtype=torch.float16)
    lse = torch.empty(B, nh, S, device=cuda_device)
    llmcu.attention_fwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), lse.data_ptr(), B, S, nh, nkv, hd,
                        nh * hd, nkv * hd, nkv * hd, st)
    assert llmcu.kernel_checks(st) == 0
    assert torch.isfinite(o.float()).all()
