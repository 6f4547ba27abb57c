"""The reference's own tests (tests/test_correctness.py and
tests/test_decode_bundle.py of the reference project), run against the drop-in
package through the reference's import name and public API.

The reference value is computed here with plain torch ops that restate
dequant_ref (focal_w4a16/__init__.py:86-91) so it does not depend on the
package under test.  Both tolerance forms are asserted: the reference's
max-abs/max-rel metric and allclose(atol=2e-2, rtol=1e-2).
"""
import sys

import pytest
import torch

import focal_w4a16

pytestmark = pytest.mark.gpu

MAX_ABS_ERR = 0.25
MAX_REL_ERR = 0.03
MIN_M1_SPEEDUP = 1.5
MIN_M1_PREDEQUANT_SPEEDUP = 1.2

SHAPES = [(M, K, N) for M in [1, 2, 4, 8] for K in [4096, 8192] for N in [4096, 8192, 11008]] + [
    (M, 11008, 4096) for M in [1, 2, 4, 8]
]
LAYERS = [("q_proj", 1, 4096, 4096), ("k_proj", 1, 4096, 4096), ("v_proj", 1, 4096, 4096),
          ("o_proj", 1, 4096, 4096), ("gate_proj", 1, 4096, 11008), ("up_proj", 1, 4096, 11008),
          ("down_proj", 1, 11008, 4096)]


def torch_dequant(wq, scales, zeros, K):
    n, kw = wq.shape
    shifts = torch.arange(8, device=wq.device, dtype=torch.int32) * 4
    q = ((wq.view(n, kw, 1) >> shifts.view(1, 1, 8)) & 0xF).to(torch.float32).reshape(n, K)
    s = scales.to(torch.float32).repeat_interleave(128, dim=1)
    z = zeros.to(torch.float32).repeat_interleave(128, dim=1)
    return (q - z) * s


def max_errors(y, ref):
    diff = (y.float() - ref.float()).abs()
    return diff.max().item(), (diff / ref.float().abs().clamp_min(1.0)).max().item()


def check(y, ref, what):
    a, r = max_errors(y, ref)
    sys.__stdout__.write(f"{what} max_abs_err={a:.6f} max_rel_err={r:.6f}\n")
    assert a <= MAX_ABS_ERR and r <= MAX_REL_ERR, what
    assert torch.allclose(y.float(), ref.float(), atol=2e-2, rtol=1e-2), what


def time_cuda(fn, warmup, iters):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(iters):
        fn()
    end.record()
    torch.cuda.synchronize()
    return start.elapsed_time(end) / iters


@pytest.mark.parametrize("M,K,N", SHAPES)
def test_w4a16_linear_correctness(cuda, M, K, N):
    x, wq, scales, zeros = focal_w4a16.random_case(M, K, N, seed=1234)
    y = focal_w4a16.w4a16_linear(x, wq, scales, zeros)
    ref = (x.float() @ torch_dequant(wq, scales, zeros, K).T).to(torch.bfloat16)
    torch.cuda.synchronize()
    check(y, ref, f"M={M} K={K} N={N}")


def test_dequant_ref_is_bit_identical_to_torch_restatement(cuda):
    x, wq, scales, zeros = focal_w4a16.random_case(8, 8192, 11008, seed=1234)
    a = focal_w4a16.dequant_ref(wq, scales, zeros, 8192)
    b = torch_dequant(wq, scales, zeros, 8192)
    assert torch.equal(a.view(torch.int32), b.view(torch.int32))


def test_unhelpful_k11008_wide_n_is_rejected(cuda):
    x = torch.empty((1, 11008), device="cuda", dtype=torch.bfloat16)
    wq = torch.empty((11008, 11008 // 8), device="cuda", dtype=torch.int32)
    scales = torch.empty((11008, 11008 // 128), device="cuda", dtype=torch.float16)
    zeros = torch.empty((11008, 11008 // 128), device="cuda", dtype=torch.float16)
    with pytest.raises(RuntimeError, match="unsupported K/N"):
        focal_w4a16.w4a16_linear(x, wq, scales, zeros)


def test_structured_pack_order_matches_direct_reference(cuda):
    M, K, N = 2, 4096, 4096
    gen = torch.Generator(device="cuda")
    gen.manual_seed(4321)
    x = 0.01 * torch.randn((M, K), device="cuda", dtype=torch.bfloat16, generator=gen)
    q = torch.arange(K, device="cuda", dtype=torch.int64).remainder(16).to(torch.uint8).repeat(N, 1).contiguous()
    wq = focal_w4a16.pack_int4_weight(q)
    scales = torch.full((N, K // 128), 0.01, device="cuda", dtype=torch.float16)
    zeros = torch.full((N, K // 128), 7.0, device="cuda", dtype=torch.float16)
    y = focal_w4a16.w4a16_linear(x.contiguous(), wq, scales, zeros)
    w_direct = (q.float() - zeros[0, 0].float()) * scales[0, 0].float()
    ref = (x.float() @ w_direct.T).to(torch.bfloat16)
    torch.cuda.synchronize()
    check(y, ref, "structured_pack")


def test_m1_kill_criterion_speed(cuda):
    M, K, N = 1, 4096, 4096
    x, wq, scales, zeros = focal_w4a16.random_case(M, K, N, seed=1234)
    w_deq = torch_dequant(wq, scales, zeros, K)
    focal_ms = time_cuda(lambda: focal_w4a16.w4a16_linear(x, wq, scales, zeros), 20, 100)
    baseline_ms = time_cuda(
        lambda: (x.float() @ torch_dequant(wq, scales, zeros, K).T).to(torch.bfloat16), 20, 100)
    predequant_ms = time_cuda(lambda: (x.float() @ w_deq.T).to(torch.bfloat16), 20, 100)
    sys.__stdout__.write(f"focal_ms={focal_ms:.6f} baseline_ms={baseline_ms:.6f} "
                         f"predequant_ms={predequant_ms:.6f}\n")
    assert baseline_ms / focal_ms >= MIN_M1_SPEEDUP
    assert predequant_ms / focal_ms >= MIN_M1_PREDEQUANT_SPEEDUP


def test_llama2_7b_supported_decode_bundle(cuda):
    for index, (name, M, K, N) in enumerate(LAYERS):
        x, wq, scales, zeros = focal_w4a16.random_case(M, K, N, seed=5000 + index)
        y = focal_w4a16.w4a16_linear(x, wq, scales, zeros)
        ref = (x.float() @ torch_dequant(wq, scales, zeros, K).T).to(torch.bfloat16)
        torch.cuda.synchronize()
        check(y, ref, name)


def test_wider_contract_shapes(cuda):
    """Shapes outside the reference's whitelist that the rule-based guard accepts."""
    for (M, K, N) in [(3, 4096, 4096), (8, 8192, 28672), (8, 28672, 8192), (5, 5120, 13824),
                      (1, 13824, 5120)]:
        g = torch.Generator(device="cuda").manual_seed(M + K + N)
        x = torch.randn((M, K), device="cuda", dtype=torch.bfloat16, generator=g)
        wq = torch.randint(-(2**31), 2**31 - 1, (N, K // 8), device="cuda", dtype=torch.int32, generator=g)
        scales = 0.005 + 0.015 * torch.rand((N, K // 128), device="cuda", generator=g).half()
        zeros = torch.randint(0, 16, (N, K // 128), device="cuda", generator=g).half()
        y = focal_w4a16.w4a16_linear(x, wq, scales, zeros)
        ref = (x.float() @ torch_dequant(wq, scales, zeros, K).T).to(torch.bfloat16)
        check(y, ref, f"M={M} K={K} N={N}")


def test_tensor_validation_messages(cuda):
    x, wq, scales, zeros = focal_w4a16.random_case(1, 4096, 4096, seed=1)
    cases = [
        ((x.cpu(), wq, scales, zeros), "x must be a CUDA tensor"),
        ((x, wq[:, ::2], scales, zeros), "wq must be contiguous"),
        ((x.float(), wq, scales, zeros), "x has wrong dtype"),
        ((x, wq, scales.float(), zeros), "scales has wrong dtype"),
        ((x[0], wq, scales, zeros), r"x must have shape \[M, K\]"),
        ((x, wq[:, :256].contiguous(), scales, zeros), r"wq must have shape \[N, K / 8\]"),
        ((x, wq, scales[:, :16].contiguous(), zeros), r"scales must have shape \[N, K / 128\]"),
        ((x, wq, scales, zeros[:2048].contiguous()), r"zeros must have shape \[N, K / 128\]"),
        ((torch.cat([x] * 9), wq, scales, zeros), "unsupported M"),
    ]
    for args, msg in cases:
        with pytest.raises(RuntimeError, match=msg):
            focal_w4a16.w4a16_linear(*args)
    with pytest.raises(ValueError, match="w_q_uint8 must be a CUDA tensor"):
        focal_w4a16.pack_int4_weight(torch.zeros((4, 8), dtype=torch.uint8))
    with pytest.raises(ValueError, match="K must be divisible by 128"):
        focal_w4a16.dequant_ref(wq, scales, zeros, 4000)
