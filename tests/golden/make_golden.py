"""Generate the golden fixtures in this folder from the reference's own code.

Run once, in a container that has the reference checkout, naming it in
FOCAL_REFERENCE_DIR (there is no default location):

    FOCAL_REFERENCE_DIR=<reference checkout> python tests/golden/make_golden.py

It imports the reference package ``focal_w4a16`` from that checkout, relaxes
its CUDA-only guard (``require_cuda_contiguous``, focal_w4a16/__init__.py:31-35)
to a contiguity check so the helpers run on CPU tensors, and records:

* ``pack.npz``       — pack_int4_weight (focal_w4a16/__init__.py:38-54) on random nibbles
                       and on hand-written known answers (README.md:66-73 formula);
* ``dequant_*.npz``  — dequant_ref (focal_w4a16/__init__.py:57-91) for both generators:
                       the benchmark one (random 32-bit words, integer zeros) and the
                       reference's random_case one (non-integer zeros 7 + U[0,1));
* ``linear_*.npz``   — baseline_dequant_matmul (bench/bench_w4a16.py:42-45):
                       (x.float() @ dequant_ref(...).T).to(bfloat16), M in {1,2,4,8};
* ``structured.npz`` — the nibble-order test of tests/test_correctness.py:83-111
                       (q = k mod 16, s = 0.01, z = 7, M=2, K=N=4096), inputs drawn on a
                       seeded CPU generator because the checkout's version needs CUDA.

bf16 tensors are stored as uint16 bit patterns.  The GPU box never runs this
script; the tests read only the .npz files.
"""
from __future__ import annotations

import importlib
import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REF_DIR = Path(os.environ["FOCAL_REFERENCE_DIR"]) if os.environ.get("FOCAL_REFERENCE_DIR") else None


def load_reference():
    if REF_DIR is None or not (REF_DIR / "focal_w4a16").is_dir():
        sys.exit("FOCAL_REFERENCE_DIR must name the reference checkout (with focal_w4a16/)")
    sys.path.insert(0, str(REF_DIR))
    try:
        ref = importlib.import_module("focal_w4a16")
    finally:
        sys.path.pop(0)
    if not str(Path(ref.__file__).resolve()).startswith(str(REF_DIR.resolve())):
        raise RuntimeError(f"imported focal_w4a16 from {ref.__file__}, not the reference")

    def contiguous_only(name, tensor):
        if not tensor.is_contiguous():
            raise ValueError(f"{name} must be contiguous")

    ref.require_cuda_contiguous = contiguous_only
    return ref


def bits(t: torch.Tensor) -> np.ndarray:
    assert t.dtype == torch.bfloat16
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def baseline_inputs(M, K, N, seed):
    """The benchmark generator on a seeded torch CPU generator."""
    g = torch.Generator(device="cpu")
    g.manual_seed(seed)
    x = torch.randn((M, K), generator=g, dtype=torch.float32).to(torch.bfloat16)
    wq = torch.randint(-(2**31), 2**31, (N, K // 8), generator=g, dtype=torch.int64).to(torch.int32)
    scales = (0.005 + 0.015 * torch.rand((N, K // 128), generator=g, dtype=torch.float32)).to(torch.float16)
    zeros = torch.randint(0, 16, (N, K // 128), generator=g, dtype=torch.int64).to(torch.float16)
    return x, wq, scales, zeros


def reference_style_inputs(ref, M, K, N, seed):
    """random_case's distributions (focal_w4a16/__init__.py:111-120) on a CPU generator."""
    g = torch.Generator(device="cpu")
    g.manual_seed(seed)
    x = torch.randn((M, K), generator=g, dtype=torch.bfloat16)
    q = torch.randint(0, 16, (N, K), generator=g, dtype=torch.uint8)
    wq = ref.pack_int4_weight(q)
    scales = 0.005 + 0.045 * torch.rand((N, K // 128), generator=g, dtype=torch.float16)
    zeros = 7.0 + torch.rand((N, K // 128), generator=g, dtype=torch.float16)
    return x, wq, scales.contiguous(), zeros.contiguous(), q


def main():
    ref = load_reference()
    torch.backends.cuda.matmul.allow_tf32 = False

    # -- packing: random nibbles (upper bits set too, to check the & 0xF) and known answers
    g = torch.Generator().manual_seed(11)
    q = torch.randint(0, 256, (64, 256), generator=g, dtype=torch.int64).to(torch.uint8)
    packed = ref.pack_int4_weight(q)
    ka_q = torch.tensor([[0, 1, 2, 3, 4, 5, 6, 7, 15, 14, 13, 12, 11, 10, 9, 8],
                         [15] * 16], dtype=torch.uint8)
    ka_packed = ref.pack_int4_weight(ka_q)
    np.savez_compressed(HERE / "pack.npz", q=q.numpy(), packed=packed.numpy(),
                        ka_q=ka_q.numpy(), ka_packed=ka_packed.numpy())

    # -- dequant, both generators
    for name, (x, wq, s, z) in {
        "baseline": baseline_inputs(1, 1024, 96, 1234),
        "refstyle": reference_style_inputs(ref, 1, 1024, 96, 1234)[:4],
    }.items():
        deq = ref.dequant_ref(wq, s, z, 1024)
        np.savez_compressed(HERE / f"dequant_{name}.npz", wq=wq.numpy(), scales=s.numpy(),
                            zeros=z.numpy(), deq=deq.numpy(), K=1024)

    # -- linear outputs (the reference's CPU baseline_dequant_matmul)
    for name, K, N in (("k512_n128", 512, 128), ("k1024_n192", 1024, 192)):
        _, wq, s, z = baseline_inputs(8, K, N, 2024)
        out = {"wq": wq.numpy(), "scales": s.numpy(), "zeros": z.numpy(), "K": K, "N": N}
        for M in (1, 2, 4, 8):
            x = baseline_inputs(M, K, N, 3000 + M)[0]
            y = (x.float() @ ref.dequant_ref(wq, s, z, K).T).to(torch.bfloat16)
            out[f"x{M}"] = bits(x)
            out[f"y{M}"] = bits(y)
        np.savez_compressed(HERE / f"linear_{name}.npz", **out)

    x, wq, s, z, _ = reference_style_inputs(ref, 4, 512, 128, 5000)
    y = (x.float() @ ref.dequant_ref(wq, s, z, 512).T).to(torch.bfloat16)
    np.savez_compressed(HERE / "linear_refstyle_m4.npz", x=bits(x), wq=wq.numpy(),
                        scales=s.numpy(), zeros=z.numpy(), y=bits(y), K=512, N=128)

    # -- structured nibble-order case (tests/test_correctness.py:83-111)
    M, K, N = 2, 4096, 4096
    g = torch.Generator().manual_seed(4321)
    x = (0.01 * torch.randn((M, K), generator=g, dtype=torch.bfloat16)).contiguous()
    qs = torch.arange(K, dtype=torch.int64).remainder(16).to(torch.uint8).repeat(N, 1).contiguous()
    wq = ref.pack_int4_weight(qs)
    s = torch.full((N, K // 128), 0.01, dtype=torch.float16)
    z = torch.full((N, K // 128), 7.0, dtype=torch.float16)
    w_direct = (qs.float() - z[0, 0].float()) * s[0, 0].float()
    y_direct = (x.float() @ w_direct.T).to(torch.bfloat16)
    y_packed = (x.float() @ ref.dequant_ref(wq, s, z, K).T).to(torch.bfloat16)
    assert torch.equal(wq[0], wq[-1])
    np.savez_compressed(HERE / "structured.npz", x=bits(x), wq_row=wq[0].numpy(),
                        y_direct=bits(y_direct), y_packed=bits(y_packed), M=M, K=K, N=N)
    for f in sorted(HERE.glob("*.npz")):
        print(f.name, f.stat().st_size)


if __name__ == "__main__":
    main()
