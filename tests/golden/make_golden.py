"""Generate tests/golden/reference_cases.pt from the reference's own math.

Run in a checkout where the reference project is available (it is not needed
to run the tests): imports ``python/cuda_operator_lab/references.py`` of the
reference by path, evaluates each of its functions on small seeded CPU inputs
that cover the edge cases the reference's tests exercise (single elements,
widths around warp/vector boundaries, odd widths, +-1000 logits, large-offset
LayerNorm rows, a K=64 GEMM in the shape family of the small benchmark GEMM), and saves inputs and outputs.

Usage: python tests/golden/make_golden.py /path/to/reference
"""

from __future__ import annotations

import importlib.util
import sys
from pathlib import Path

import torch

OUT = Path(__file__).resolve().parent / "reference_cases.pt"


def load_references(reference_root: Path):
    path = reference_root / "python" / "cuda_operator_lab" / "references.py"
    spec = importlib.util.spec_from_file_location("reference_references", path)
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    return module


def gen(seed: int) -> torch.Generator:
    g = torch.Generator(device="cpu")
    g.manual_seed(seed)
    return g


def randn(g, *shape, scale=1.0, offset=0.0):
    return torch.randn(*shape, generator=g, dtype=torch.float32) * scale + offset


def bf16(g, *shape, scale=1.0):
    return (torch.randn(*shape, generator=g, dtype=torch.float32) * scale).to(torch.bfloat16)


def build_cases(ref) -> list[dict]:
    cases: list[dict] = []

    def add(fn: str, args: list, kwargs: dict | None = None, tag: str = "") -> None:
        kwargs = kwargs or {}
        expected = getattr(ref, fn)(*args, **kwargs)
        cases.append({"fn": fn, "tag": tag, "args": args, "kwargs": kwargs, "expected": expected})

    # reduction_sum (references.py:8-14); seeds follow the reference tests' 20261004 + n
    add("reduction_sum", [torch.arange(1, 1026, dtype=torch.float32)], tag="arange_1_1025")
    for n in (1, 2, 33, 1025, 16385):
        add("reduction_sum", [torch.rand(n, generator=gen(20261004 + n), dtype=torch.float32)],
            tag=f"rand_{n}")
    add("reduction_sum", [torch.rand(65539, generator=gen(7), dtype=torch.float32) * 2 - 1],
        tag="uniform_pm1_65539")

    # row_softmax (references.py:17-25)
    add("row_softmax", [torch.tensor([[1000.0, 1001.0, 999.0, 998.0],
                                      [-1000.0, -999.0, -1001.0, -1002.0]])], tag="large_logits")
    for rows, cols in ((1, 1), (1, 3), (2, 33), (7, 513), (2, 4097), (2, 4096)):
        g = gen(20261005 + rows * 10000 + cols)
        add("row_softmax", [randn(g, rows, cols, scale=2.0)], tag=f"{rows}x{cols}")

    # rmsnorm (references.py:28-47)
    add("rmsnorm", [torch.tensor([[1000.0, -1000.0, 500.0, -500.0]]),
                    torch.tensor([1.0, 0.5, -2.0, 3.0])], tag="pm1000_signed_weight")
    for rows, cols, eps in ((1, 1, 1e-5), (2, 33, 1e-5), (7, 127, 1e-6), (2, 4097, 1e-5),
                            (1, 8192, 1e-6)):
        g = gen(20261005 + rows * 10000 + cols)
        x = randn(g, rows, cols)
        w = torch.rand(cols, generator=g, dtype=torch.float32) + 0.5
        add("rmsnorm", [x, w], {"eps": eps}, tag=f"{rows}x{cols}_eps{eps:g}")

    # layernorm (references.py:50-77)
    g = gen(20261005)
    add("layernorm", [randn(g, 4, 4096, scale=0.1, offset=1000.0), randn(g, 4096), randn(g, 4096)],
        tag="offset_1000")
    for rows, cols in ((1, 1), (2, 33), (17, 1024), (7, 127), (3, 4097)):
        g = gen(20261005 + rows * 10000 + cols)
        add("layernorm", [randn(g, rows, cols), torch.rand(cols, generator=g) + 0.5,
                          randn(g, cols, scale=0.1)], tag=f"{rows}x{cols}")

    # fused_residual_layernorm (references.py:80-98)
    for rows, cols in ((1, 1), (7, 127), (2, 4097), (1, 4096)):
        g = gen(20261006 + rows * 10000 + cols)
        add("fused_residual_layernorm",
            [randn(g, rows, cols), randn(g, rows, cols), torch.rand(cols, generator=g) + 0.5,
             randn(g, cols, scale=0.1)], tag=f"{rows}x{cols}")

    # fused_bias_gelu (references.py:101-112) and swiglu (:115-121)
    for rows, cols in ((1, 1), (17, 31), (64, 256), (3, 4096)):
        g = gen(20261007 + rows * 10000 + cols)
        add("fused_bias_gelu", [randn(g, rows, cols, scale=2.0), randn(g, cols, scale=0.1)],
            tag=f"{rows}x{cols}")
        g = gen(20261008 + rows * 10000 + cols)
        add("swiglu", [randn(g, rows, cols, scale=3.0), randn(g, rows, cols)], tag=f"{rows}x{cols}")
    add("swiglu", [torch.tensor([-100.0, -20.0, -1.0, 0.0, 1.0, 20.0, 100.0]),
                   torch.ones(7)], tag="extremes")

    # fp32 GEMM epilogues (references.py:124-200)
    for m, k, n in ((1, 1, 1), (4, 16, 32), (17, 31, 63)):
        g = gen(20261005 + m * 1000000 + k * 1000 + n)
        x, w, b = randn(g, m, k), randn(g, n, k), randn(g, n)
        add("gemm_bias_gelu", [x, w, b], tag=f"{m}x{k}x{n}")
        add("gemm_bias_gelu_tanh", [x, w, b], tag=f"{m}x{k}x{n}")
        g = gen(20261010 + m * 1000000 + k * 1000 + n)
        x, wg, wu = randn(g, m, k), randn(g, n, k), randn(g, n, k)
        add("gemm_swiglu", [x, wg, wu], tag=f"{m}x{k}x{n}")
        add("gemm_swiglu_packed", [x, torch.cat((wg, wu), dim=0)], tag=f"{m}x{k}x{n}")

    # bf16 GEMM+SwiGLU references (references.py:203-271)
    for m, k, n in ((16, 64, 64), (32, 128, 256), (17, 40, 24), (64, 64, 512)):
        g = gen(20261025 + m * 1000000 + k * 1000 + n)
        x = bf16(g, m, k)
        wg, wu = bf16(g, n, k, scale=k ** -0.5), bf16(g, n, k, scale=k ** -0.5)
        packed = torch.cat((wg, wu), dim=0).contiguous()
        add("gemm_swiglu_bf16_fp32_reference", [x, packed], tag=f"{m}x{k}x{n}")
        add("gemm_swiglu_bf16_dual_fp32_reference", [x, wg, wu], tag=f"{m}x{k}x{n}")
        if m * n <= 8192:
            add("gemm_swiglu_bf16_workspace_reference", [x, packed], tag=f"{m}x{k}x{n}")
    return cases


def main() -> None:
    if len(sys.argv) != 2:
        raise SystemExit(__doc__)
    ref = load_references(Path(sys.argv[1]))
    torch.manual_seed(0)
    torch.set_num_threads(1)
    cases = build_cases(ref)
    torch.save({"source": "python/cuda_operator_lab/references.py", "torch": str(torch.__version__),
                "cases": cases}, OUT)
    print(f"wrote {len(cases)} cases to {OUT} ({OUT.stat().st_size / 1e6:.2f} MB)")


if __name__ == "__main__":
    main()
