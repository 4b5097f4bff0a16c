"""Host-side contract of the bindings that needs no GPU (CPU).

Every public op rejects CPU tensors with a ValueError naming CUDA before it
touches the library, as the reference bindings do (e.g. reference
bindings.py:441-444; tests/test_reduction_v0.py:27-29).
"""

from __future__ import annotations

import inspect

import pytest
import torch

from cuda_operator_lab import bindings as b


def _cpu_args(name: str):
    f32 = lambda *s: torch.zeros(*s, dtype=torch.float32)  # noqa: E731
    bf = lambda *s: torch.zeros(*s, dtype=torch.bfloat16)  # noqa: E731
    if name == "rmsnorm_allgather_bf16":
        return [bf(2, 8), bf(8), [1 << 20]]
    if name.startswith("reduction"):
        return [f32(8)]
    if name.startswith("softmax"):
        return [f32(2, 8)]
    if name.startswith("rmsnorm_bf16"):
        return [bf(2, 8), bf(8)]
    if name.startswith("rmsnorm"):
        return [f32(2, 8), f32(8)]
    if name.startswith("layernorm"):
        return [f32(2, 8), f32(8), f32(8)]
    if name.startswith("fused_residual_rmsnorm"):
        return [f32(2, 8), f32(2, 8), f32(8)]
    if name.startswith("fused_residual_layernorm"):
        return [f32(2, 8), f32(2, 8), f32(8), f32(8)]
    if name.startswith("fused_bias_gelu"):
        return [f32(2, 8), f32(8)]
    if name.startswith("swiglu"):
        return [f32(2, 8), f32(2, 8)]
    if name.startswith("rmsnorm_rstd_bf16"):
        return [bf(2, 8)]
    if name == "gemm_swiglu_allgather_bf16":
        return [bf(2, 8), None, bf(8, 8), [1 << 20], 4]
    if name.startswith("gemm_swiglu_rowscale_bf16"):
        return [bf(2, 8), f32(2), bf(8, 8)]
    if name.startswith("gemm_residual_bf16"):
        return [bf(2, 8), bf(4, 8), bf(2, 4)]
    if name.startswith("gemm_bias_gelu_bf16"):
        return [bf(2, 8), bf(4, 8), f32(4)]
    if name.startswith("gemm_bias_gelu"):
        return [f32(2, 8), f32(4, 8), f32(4)]
    if name == "gemm_swiglu_bf16":
        return [bf(2, 8), bf(8, 8)]
    if name in ("gemm_swiglu_v0", "gemm_swiglu_v1"):
        return [f32(2, 8), f32(4, 8), f32(4, 8)]
    if name in ("gemm_swiglu_v2", "gemm_swiglu_v3"):
        return [f32(2, 8), f32(8, 8)]
    if name in ("gemm_swiglu_v4", "gemm_swiglu_v5", "gemm_swiglu_v10", "gemm_swiglu_v11"):
        return [bf(2, 16), bf(32, 16)]
    if name.startswith("gemm_swiglu_v"):
        return [bf(16, 16), bf(64, 16), bf(64, 16)]
    raise KeyError(name)


ALLOCATING_OPS = sorted(
    name for name in b.__all__
    if not name.endswith("_into") and callable(getattr(b, name))
    and name not in ("gemm_status", "device_info", "build_tag", "library_path",
                     "fold_rmsnorm_weight", "peer_alloc", "peer_open", "peer_close",
                     "peer_free", "peer_barrier", "peer_status")
)


def test_every_reference_operator_is_exported():
    families = {
        "reduction": 6, "softmax": 6, "rmsnorm": 5, "layernorm": 6,
        "fused_residual_layernorm": 5, "fused_bias_gelu": 3, "swiglu": 3,
        "gemm_bias_gelu": 7, "gemm_swiglu": 12,
    }
    for family, count in families.items():
        for v in range(12):
            present = hasattr(b, f"{family}_v{v}") and hasattr(b, f"{family}_v{v}_into")
            if family == "gemm_swiglu":
                assert present == (v < count), (family, v)
            else:
                assert present == (v < count), (family, v)


@pytest.mark.parametrize("name", ALLOCATING_OPS)
def test_cpu_tensors_are_rejected_before_the_library(name: str):
    fn = getattr(b, name)
    with pytest.raises(ValueError, match="CUDA"):
        fn(*_cpu_args(name))


def test_into_signatures_match_reference_argument_order():
    sig = inspect.signature(b.rmsnorm_v4_into)
    assert list(sig.parameters) == ["x", "weight", "out", "eps"]
    assert sig.parameters["eps"].default == 1e-5
    sig = inspect.signature(b.fused_residual_layernorm_v2_into)
    assert list(sig.parameters) == ["x", "residual", "weight", "bias", "out", "eps"]
    sig = inspect.signature(b.gemm_swiglu_v11_into)
    assert list(sig.parameters) == ["x", "packed_weight", "workspace", "out"]
    sig = inspect.signature(b.gemm_swiglu_v7_into)
    assert list(sig.parameters) == ["x_bf16", "gate_weight_bf16", "up_weight_bf16", "out"]


def test_missing_library_fails_loudly(tmp_path, monkeypatch):
    monkeypatch.setenv("CUDA_OPERATOR_LIB", str(tmp_path / "absent.so"))
    monkeypatch.setattr(b, "_LIBRARY", None)
    with pytest.raises(RuntimeError, match="not found"):
        b._library()


def test_peer_barrier_rank_checks_before_the_library():
    for addrs, rank in (([], 0), ([1] * 9, 0), ([1, 2], 2), ([1], -1)):
        with pytest.raises(ValueError):
            b.peer_barrier(addrs, rank, 1)
