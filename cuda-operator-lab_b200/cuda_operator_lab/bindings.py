"""ctypes bindings for the sm_100a operator library (drop-in for the reference).

Same public functions, arguments, validation messages, stream semantics and
return conventions as the reference module ``python/cuda_operator_lab/
bindings.py`` (its line numbers are cited per family below): every
``<op>_v<k>_into`` validates PyTorch CUDA tensors on the host, passes their
raw device pointers and ``torch.cuda.current_stream(x.device)`` to one
``extern "C"`` symbol of ``libcuda_operator_lab.so`` (declared in
``include/cuda_operator_lab.h``) and raises ``RuntimeError("CUDA error
{code}: {message}")`` on a non-zero return; ``<op>_v<k>`` allocates the
output and calls ``_into``.

There is no fallback: if the shared library is missing, the first call raises
``RuntimeError``.  ``CUDA_OPERATOR_LIB`` overrides the library path
(reference ``bindings.py:17-21``).

Functions after the reference set (``rmsnorm_bf16``, ``fused_residual_layernorm_h``,
``fused_residual_rmsnorm``, ``gemm_swiglu_bf16``, ``gemm_bias_gelu_bf16``,
``gemm_residual_bf16``, ``rmsnorm_rstd_bf16``, ``gemm_swiglu_rowscale_bf16``,
``gemm_swiglu_allgather_bf16``, ``reduction_partial_f64``, ``peer_*``) expose the
library's additional entry points.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path
from typing import Callable, Sequence

import torch

__all__: list[str] = []

# ---------------------------------------------------------------- library

_P = ctypes.c_void_p
_U64 = ctypes.c_uint64
_F32 = ctypes.c_float
_I32 = ctypes.c_int

# symbol -> argtypes (restype int unless listed in _RESTYPES)
_SIGNATURES: dict[str, list] = {}
for _v in range(6):
    _SIGNATURES[f"cuda_operator_reduction_v{_v}"] = [_P, _P, _U64, _P]
    _SIGNATURES[f"cuda_operator_softmax_v{_v}"] = [_P, _P, _U64, _U64, _P]
    _SIGNATURES[f"cuda_operator_layernorm_v{_v}"] = [_P, _P, _P, _P, _U64, _U64, _F32, _P]
for _v in range(5):
    _SIGNATURES[f"cuda_operator_rmsnorm_v{_v}"] = [_P, _P, _P, _U64, _U64, _F32, _P]
    _SIGNATURES[f"cuda_operator_fused_residual_layernorm_v{_v}"] = [
        _P, _P, _P, _P, _P, _U64, _U64, _F32, _P]
for _v in range(3):
    _SIGNATURES[f"cuda_operator_fused_bias_gelu_v{_v}"] = [_P, _P, _P, _U64, _U64, _P]
_SIGNATURES["cuda_operator_swiglu_v0"] = [_P, _P, _P, _U64, _P]
_SIGNATURES["cuda_operator_swiglu_v1"] = [_P, _P, _P, _U64, _P]
_SIGNATURES["cuda_operator_swiglu_v2"] = [_P, _P, _P, _U64, _U64, _P]
for _v in range(7):
    _SIGNATURES[f"cuda_operator_gemm_bias_gelu_v{_v}"] = [_P, _P, _P, _P, _U64, _U64, _U64, _P]
for _v in (0, 1):
    _SIGNATURES[f"cuda_operator_gemm_swiglu_v{_v}"] = [_P, _P, _P, _P, _P, _U64, _U64, _U64, _P]
for _v in (2, 3, 4, 5, 10, 11):
    _SIGNATURES[f"cuda_operator_gemm_swiglu_v{_v}"] = [_P, _P, _P, _P, _U64, _U64, _U64, _P]
for _v in (6, 7, 8, 9):
    _SIGNATURES[f"cuda_operator_gemm_swiglu_v{_v}"] = [_P, _P, _P, _P, _U64, _U64, _U64, _P]
_SIGNATURES["cuda_operator_error_string"] = [_I32]
# entry points new in this library
_SIGNATURES["cuda_operator_rmsnorm_bf16"] = [_P, _P, _P, _U64, _U64, _F32, _P]
_SIGNATURES["cuda_operator_fused_residual_layernorm_h"] = [
    _P, _P, _P, _P, _P, _P, _U64, _U64, _F32, _P]
_SIGNATURES["cuda_operator_fused_residual_rmsnorm_bf16"] = [
    _P, _P, _P, _P, _P, _U64, _U64, _F32, _P]
_SIGNATURES["cuda_operator_fused_residual_rmsnorm_h"] = [_P, _P, _P, _P, _P, _U64, _U64, _F32, _P]
_SIGNATURES["cuda_operator_gemm_swiglu_bf16"] = [_P, _P, _P, _U64, _U64, _U64, _P]
_SIGNATURES["cuda_operator_gemm_bias_gelu_bf16"] = [_P, _P, _P, _P, _U64, _U64, _U64, _P]
_SIGNATURES["cuda_operator_gemm_residual_bf16"] = [_P, _P, _P, _P, _U64, _U64, _U64, _P]
_SIGNATURES["cuda_operator_rmsnorm_rstd_bf16"] = [_P, _P, _U64, _U64, _F32, _P]
_SIGNATURES["cuda_operator_gemm_swiglu_rowscale_bf16"] = [_P, _P, _P, _P, _U64, _U64, _U64, _P]
_SIGNATURES["cuda_operator_gemm_swiglu_allgather_bf16"] = [
    _P, _P, _P, _P, _I32, _U64, _U64, _U64, _U64, _P]
_SIGNATURES["cuda_operator_rmsnorm_allgather_bf16"] = [_P, _P, _P, _I32, _U64, _U64, _F32, _P]
_SIGNATURES["cuda_operator_reduction_partial_f64"] = [_P, _P, _U64, _P]
_SIGNATURES["cuda_operator_lab_peer_handle_bytes"] = []
_SIGNATURES["cuda_operator_lab_peer_alloc"] = [_U64, _P, _P]
_SIGNATURES["cuda_operator_lab_peer_open"] = [_P, _P]
_SIGNATURES["cuda_operator_lab_peer_close"] = [_P]
_SIGNATURES["cuda_operator_lab_peer_free"] = [_P]
_SIGNATURES["cuda_operator_lab_peer_barrier"] = [_P, _I32, _I32, ctypes.c_uint32, _U64, _P]
_SIGNATURES["cuda_operator_lab_peer_status"] = [_P, _I32]
_SIGNATURES["cuda_operator_lab_device_info"] = [_P, _P, _P]
_SIGNATURES["cuda_operator_lab_build_tag"] = []
_SIGNATURES["cuda_operator_lab_gemm_status"] = [_P, _I32]
_SIGNATURES["cuda_operator_lab_reduction_noalloc"] = [_P, _P, _U64, _P]

_RESTYPES = {
    "cuda_operator_error_string": ctypes.c_char_p,
    "cuda_operator_lab_peer_handle_bytes": ctypes.c_uint64,
    "cuda_operator_lab_build_tag": ctypes.c_char_p,
}

#: The 54 symbols of the reference library (``bindings.py:32-417``).
REFERENCE_SYMBOLS = tuple(
    name for name in _SIGNATURES
    if name == "cuda_operator_error_string"
    or (name.startswith("cuda_operator_") and name.rsplit("_", 1)[-1][:1] == "v"
        and name.rsplit("_", 1)[-1][1:].isdigit())
)


def _default_library_path() -> Path:
    override = os.environ.get("CUDA_OPERATOR_LIB")
    if override:
        return Path(override).expanduser().resolve()
    return Path(__file__).resolve().parents[1] / "build" / "lib" / "libcuda_operator_lab.so"


class _Library:
    """The loaded shared library with argtypes declared for every symbol.

    Like the reference (``bindings.py:24-31``) every symbol is resolved
    eagerly, so a library that lacks one fails at load time, not mid-run.
    """

    def __init__(self, path: Path, symbols: tuple[str, ...] | None = None) -> None:
        if not path.is_file():
            raise RuntimeError(
                f"CUDA operator library not found at {path}. "
                "Build it with `python cuda-operator-lab_b200/build.py`."
            )
        self.path = path
        self.handle = ctypes.CDLL(str(path))
        self.functions: dict[str, Callable] = {}
        for name in symbols if symbols is not None else tuple(_SIGNATURES):
            function = getattr(self.handle, name)
            function.argtypes = _SIGNATURES[name]
            function.restype = _RESTYPES.get(name, ctypes.c_int)
            self.functions[name] = function

    def check(self, code: int) -> None:
        if code == 0:
            return
        message = self.handle.cuda_operator_error_string(code)
        decoded = message.decode("utf-8", errors="replace") if message else "unknown CUDA error"
        raise RuntimeError(f"CUDA error {code}: {decoded}")


_LIBRARY: _Library | None = None


def _library() -> _Library:
    global _LIBRARY
    if _LIBRARY is None:
        _LIBRARY = _Library(_default_library_path())
    return _LIBRARY


def library_path() -> Path:
    """Path of the shared library the bindings load."""
    return _default_library_path()


# The per-call host path is kept short (a single GEMM call is launch-bound):
# pointers and sizes go to ctypes as plain ints (the declared argtypes convert
# them), the current stream is read as a raw handle without building a
# torch.cuda.Stream object, and each symbol's function object is looked up
# once and kept.
try:
    from torch._C import _cuda_getCurrentRawStream as _raw_stream
except ImportError:  # pragma: no cover - older torch
    _raw_stream = None


def _ptr(t: torch.Tensor) -> int:
    return t.data_ptr()


def _stream(t: torch.Tensor) -> int:
    if _raw_stream is not None:
        return _raw_stream(t.get_device())
    return torch.cuda.current_stream(device=t.device).cuda_stream


def _all_cuda(*tensors: torch.Tensor) -> bool:
    for t in tensors:
        if not t.is_cuda:
            return False
    return True


def _all_contiguous(*tensors: torch.Tensor) -> bool:
    for t in tensors:
        if not t.is_contiguous():
            return False
    return True


def _any_not_dtype(dtype: torch.dtype, *tensors: torch.Tensor) -> bool:
    for t in tensors:
        if t.dtype != dtype:
            return True
    return False


def _call(symbol: str, *args) -> None:
    library = _LIBRARY if _LIBRARY is not None else _library()
    code = library.functions[symbol](*args)
    if code:
        library.check(code)


def _export(name: str, fn: Callable, doc: str) -> Callable:
    fn.__name__ = name
    fn.__qualname__ = name
    fn.__doc__ = doc
    globals()[name] = fn
    __all__.append(name)
    return fn


# ---------------------------------------------------------------- reduction
# reference bindings.py:441-535


def _validate_reduction_input(x: torch.Tensor) -> None:
    if not x.is_cuda:
        raise ValueError("reduction input must be a CUDA tensor")
    if x.ndim != 1:
        raise ValueError("reduction input must be 1-D")
    if x.dtype != torch.float32:
        raise TypeError("reduction currently supports float32 only")
    if not x.is_contiguous():
        raise ValueError("reduction input must be contiguous")


def _validate_reduction_output(x: torch.Tensor, out: torch.Tensor) -> None:
    if not out.is_cuda or out.device != x.device:
        raise ValueError("output must be a CUDA tensor on the same device")
    if out.dtype != torch.float32 or out.numel() != 1 or not out.is_contiguous():
        raise ValueError("output must be one contiguous float32 CUDA value")


def _make_reduction(version: int) -> None:
    symbol = f"cuda_operator_reduction_v{version}"

    def into(x: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        _validate_reduction_input(x)
        _validate_reduction_output(x, out)
        _call(symbol, _ptr(x) if x.numel() else None, _ptr(out),
              int(x.numel()), _stream(x))
        return out

    def alloc(x: torch.Tensor) -> torch.Tensor:
        return into(x, torch.empty(1, device=x.device, dtype=torch.float32))

    doc = (f"Global fp32 sum into a one-element tensor (reference reduction_v{version}); "
           "fp64 accumulation with a fixed, run-to-run reproducible combine order.")
    _export(f"reduction_v{version}_into", into, doc)
    _export(f"reduction_v{version}", alloc, doc)


for _v in range(6):
    _make_reduction(_v)


def reduction_partial_f64_into(x: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
    """fp64 partial sum of a 1-D fp32 CUDA tensor into a one-element float64 tensor.

    The per-rank step of the multi-GPU reduction: each rank sums its chunk,
    then an all-reduce of the float64 partials forms the global sum.
    """
    _validate_reduction_input(x)
    if not out.is_cuda or out.device != x.device:
        raise ValueError("output must be a CUDA tensor on the same device")
    if out.dtype != torch.float64 or out.numel() != 1 or not out.is_contiguous():
        raise ValueError("output must be one contiguous float64 CUDA value")
    _call("cuda_operator_reduction_partial_f64", _ptr(x) if x.numel() else None,
          _ptr(out), int(x.numel()), _stream(x))
    return out


def reduction_partial_f64(x: torch.Tensor) -> torch.Tensor:
    """Allocating form of :func:`reduction_partial_f64_into`."""
    return reduction_partial_f64_into(x, torch.empty(1, device=x.device, dtype=torch.float64))


__all__ += ["reduction_partial_f64_into", "reduction_partial_f64"]

# ---------------------------------------------------------------- softmax
# reference bindings.py:538-649


def _validate_softmax_input(x: torch.Tensor) -> None:
    if not x.is_cuda:
        raise ValueError("softmax input must be a CUDA tensor")
    if x.ndim != 2:
        raise ValueError("softmax input must be 2-D [rows, cols]")
    if x.dtype != torch.float32:
        raise TypeError("softmax currently supports float32 only")
    if not x.is_contiguous():
        raise ValueError("softmax input must be contiguous")
    if x.shape[1] == 0:
        raise ValueError("softmax requires cols > 0")


def _validate_softmax_output(x: torch.Tensor, out: torch.Tensor) -> None:
    if not out.is_cuda or out.device != x.device:
        raise ValueError("softmax output must be a CUDA tensor on the same device")
    if out.dtype != torch.float32 or out.shape != x.shape or not out.is_contiguous():
        raise ValueError("softmax output must be contiguous float32 with the same shape")


def _make_softmax(version: int) -> None:
    symbol = f"cuda_operator_softmax_v{version}"

    def into(x: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        _validate_softmax_input(x)
        _validate_softmax_output(x, out)
        rows, cols = x.shape
        if rows == 0:
            return out
        _call(symbol, _ptr(x), _ptr(out), int(rows), int(cols), _stream(x))
        return out

    def alloc(x: torch.Tensor) -> torch.Tensor:
        return into(x, torch.empty_like(x))

    doc = f"Row-wise fp32 softmax (reference softmax_v{version})."
    _export(f"softmax_v{version}_into", into, doc)
    _export(f"softmax_v{version}", alloc, doc)


for _v in range(6):
    _make_softmax(_v)

# ---------------------------------------------------------------- RMSNorm
# reference bindings.py:652-873


def _validate_rmsnorm_input(x: torch.Tensor, weight: torch.Tensor, eps: float,
                            dtype: torch.dtype = torch.float32) -> None:
    if not x.is_cuda or not weight.is_cuda:
        raise ValueError("rmsnorm input and weight must be CUDA tensors")
    if x.ndim != 2:
        raise ValueError("rmsnorm input must be 2-D [rows, cols]")
    if weight.ndim != 1 or weight.shape[0] != x.shape[1]:
        raise ValueError("rmsnorm weight must be 1-D with length equal to cols")
    if x.dtype != dtype or weight.dtype != dtype:
        if dtype == torch.float32:
            raise TypeError("rmsnorm currently supports float32 only")
        raise TypeError("rmsnorm_bf16 expects bfloat16 input and weight")
    if not x.is_contiguous() or not weight.is_contiguous():
        raise ValueError("rmsnorm input and weight must be contiguous")
    if x.shape[1] == 0:
        raise ValueError("rmsnorm requires cols > 0")
    if eps <= 0:
        raise ValueError("rmsnorm eps must be positive")


def _validate_rmsnorm_output(x: torch.Tensor, out: torch.Tensor) -> None:
    if not out.is_cuda or out.device != x.device:
        raise ValueError("rmsnorm output must be a CUDA tensor on the same device")
    if out.dtype != x.dtype or out.shape != x.shape or not out.is_contiguous():
        if x.dtype == torch.float32:
            raise ValueError("rmsnorm output must be contiguous float32 with the same shape")
        raise ValueError("rmsnorm output must be contiguous bfloat16 with the same shape")


def _make_rmsnorm(version: int) -> None:
    symbol = f"cuda_operator_rmsnorm_v{version}"

    def into(x: torch.Tensor, weight: torch.Tensor, out: torch.Tensor,
             eps: float = 1e-5) -> torch.Tensor:
        _validate_rmsnorm_input(x, weight, eps)
        _validate_rmsnorm_output(x, out)
        rows, cols = x.shape
        if rows == 0:
            return out
        _call(symbol, _ptr(x), _ptr(weight), _ptr(out), int(rows),
              int(cols), float(eps), _stream(x))
        return out

    def alloc(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-5) -> torch.Tensor:
        return into(x, weight, torch.empty_like(x), eps)

    doc = f"Row-wise fp32 RMSNorm x*rsqrt(mean(x^2)+eps)*w (reference rmsnorm_v{version})."
    _export(f"rmsnorm_v{version}_into", into, doc)
    _export(f"rmsnorm_v{version}", alloc, doc)


for _v in range(5):
    _make_rmsnorm(_v)


def rmsnorm_bf16_into(x: torch.Tensor, weight: torch.Tensor, out: torch.Tensor,
                      eps: float = 1e-5) -> torch.Tensor:
    """bf16 RMSNorm with fp32 statistics: out = bf16(x * rsqrt(mean(x^2)+eps) * w)."""
    _validate_rmsnorm_input(x, weight, eps, torch.bfloat16)
    _validate_rmsnorm_output(x, out)
    rows, cols = x.shape
    if rows == 0:
        return out
    _call("cuda_operator_rmsnorm_bf16", _ptr(x), _ptr(weight), _ptr(out), int(rows),
          int(cols), float(eps), _stream(x))
    return out


def rmsnorm_bf16(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-5) -> torch.Tensor:
    """Allocating form of :func:`rmsnorm_bf16_into`."""
    return rmsnorm_bf16_into(x, weight, torch.empty_like(x), eps)


__all__ += ["rmsnorm_bf16_into", "rmsnorm_bf16"]


def fused_residual_rmsnorm_into(x: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor,
                                h_out: torch.Tensor, out: torch.Tensor,
                                eps: float = 1e-5) -> tuple[torch.Tensor, torch.Tensor]:
    """Residual add + RMSNorm in one pass: h_out = x + residual, out = rmsnorm(h) * weight.

    float32 or bfloat16 (all tensors the same dtype); for bfloat16, h is rounded
    to bfloat16 before the statistics, as a separate add would store it.
    """
    dtype = x.dtype if x.dtype in (torch.float32, torch.bfloat16) else torch.float32
    _validate_rmsnorm_input(x, weight, eps, dtype)
    if not residual.is_cuda or residual.shape != x.shape or residual.dtype != x.dtype \
            or not residual.is_contiguous():
        raise ValueError("rmsnorm residual must be a contiguous CUDA tensor shaped like the input")
    _validate_rmsnorm_output(x, out)
    _validate_rmsnorm_output(x, h_out)
    rows, cols = x.shape
    if rows == 0:
        return h_out, out
    symbol = ("cuda_operator_fused_residual_rmsnorm_bf16" if dtype == torch.bfloat16
              else "cuda_operator_fused_residual_rmsnorm_h")
    _call(symbol, _ptr(x), _ptr(residual), _ptr(weight), _ptr(h_out), _ptr(out),
          int(rows), int(cols), float(eps), _stream(x))
    return h_out, out


def fused_residual_rmsnorm(x: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor,
                           eps: float = 1e-5) -> tuple[torch.Tensor, torch.Tensor]:
    """Allocating form of :func:`fused_residual_rmsnorm_into`; returns (h, y)."""
    return fused_residual_rmsnorm_into(x, residual, weight, torch.empty_like(x),
                                       torch.empty_like(x), eps)


__all__ += ["fused_residual_rmsnorm_into", "fused_residual_rmsnorm"]

# ---------------------------------------------------------------- LayerNorm
# reference bindings.py:875-1151


def _validate_layernorm_input(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor,
                              eps: float) -> None:
    if not x.is_cuda or not weight.is_cuda or not bias.is_cuda:
        raise ValueError("layernorm input, weight, and bias must be CUDA tensors")
    if x.ndim != 2:
        raise ValueError("layernorm input must be 2-D [rows, cols]")
    if weight.ndim != 1 or weight.shape[0] != x.shape[1]:
        raise ValueError("layernorm weight must be 1-D with length equal to cols")
    if bias.ndim != 1 or bias.shape[0] != x.shape[1]:
        raise ValueError("layernorm bias must be 1-D with length equal to cols")
    if x.dtype != torch.float32 or weight.dtype != torch.float32 or bias.dtype != torch.float32:
        raise TypeError("layernorm currently supports float32 only")
    if not x.is_contiguous() or not weight.is_contiguous() or not bias.is_contiguous():
        raise ValueError("layernorm input, weight, and bias must be contiguous")
    if x.shape[1] == 0:
        raise ValueError("layernorm requires cols > 0")
    if eps <= 0:
        raise ValueError("layernorm eps must be positive")


def _validate_layernorm_output(x: torch.Tensor, out: torch.Tensor) -> None:
    if not out.is_cuda or out.device != x.device:
        raise ValueError("layernorm output must be a CUDA tensor on the same device")
    if out.dtype != torch.float32 or out.shape != x.shape or not out.is_contiguous():
        raise ValueError("layernorm output must be contiguous float32 with the same shape")


def _make_layernorm(version: int) -> None:
    symbol = f"cuda_operator_layernorm_v{version}"

    def into(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor, out: torch.Tensor,
             eps: float = 1e-5) -> torch.Tensor:
        _validate_layernorm_input(x, weight, bias, eps)
        _validate_layernorm_output(x, out)
        rows, cols = x.shape
        if rows == 0:
            return out
        _call(symbol, _ptr(x), _ptr(weight), _ptr(bias), _ptr(out), int(rows),
              int(cols), float(eps), _stream(x))
        return out

    def alloc(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor,
              eps: float = 1e-5) -> torch.Tensor:
        return into(x, weight, bias, torch.empty_like(x), eps)

    doc = f"Row-wise fp32 LayerNorm, biased variance (reference layernorm_v{version})."
    _export(f"layernorm_v{version}_into", into, doc)
    _export(f"layernorm_v{version}", alloc, doc)


for _v in range(6):
    _make_layernorm(_v)

# ---------------------------------------------------------------- residual + LayerNorm
# reference bindings.py:1154-1391


def _validate_fused_residual_layernorm_input(x: torch.Tensor, residual: torch.Tensor,
                                             weight: torch.Tensor, bias: torch.Tensor,
                                             eps: float) -> None:
    if not x.is_cuda or not residual.is_cuda or not weight.is_cuda or not bias.is_cuda:
        raise ValueError("all fused residual layernorm inputs must be CUDA tensors")
    if x.ndim != 2 or residual.shape != x.shape:
        raise ValueError("x and residual must have the same 2-D shape")
    if weight.ndim != 1 or weight.shape[0] != x.shape[1]:
        raise ValueError("weight must be 1-D with length equal to cols")
    if bias.ndim != 1 or bias.shape[0] != x.shape[1]:
        raise ValueError("bias must be 1-D with length equal to cols")
    if _any_not_dtype(torch.float32, x, residual, weight, bias):
        raise TypeError("fused residual layernorm currently supports float32 only")
    if not _all_contiguous(x, residual, weight, bias):
        raise ValueError("all fused residual layernorm inputs must be contiguous")
    if x.shape[1] == 0:
        raise ValueError("fused residual layernorm requires cols > 0")
    if eps <= 0:
        raise ValueError("eps must be positive")


def _make_residual_layernorm(version: int) -> None:
    symbol = f"cuda_operator_fused_residual_layernorm_v{version}"

    def into(x: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor,
             out: torch.Tensor, eps: float = 1e-5) -> torch.Tensor:
        _validate_fused_residual_layernorm_input(x, residual, weight, bias, eps)
        _validate_layernorm_output(x, out)
        rows, cols = x.shape
        if rows == 0:
            return out
        _call(symbol, _ptr(x), _ptr(residual), _ptr(weight), _ptr(bias), _ptr(out),
              int(rows), int(cols), float(eps), _stream(x))
        return out

    def alloc(x: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor,
              eps: float = 1e-5) -> torch.Tensor:
        return into(x, residual, weight, bias, torch.empty_like(x), eps)

    doc = (f"LayerNorm(x + residual), fp32; h itself is not stored "
           f"(reference fused_residual_layernorm_v{version}).")
    _export(f"fused_residual_layernorm_v{version}_into", into, doc)
    _export(f"fused_residual_layernorm_v{version}", alloc, doc)


for _v in range(5):
    _make_residual_layernorm(_v)


def fused_residual_layernorm_h_into(x: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor,
                                    bias: torch.Tensor, h_out: torch.Tensor, out: torch.Tensor,
                                    eps: float = 1e-5) -> tuple[torch.Tensor, torch.Tensor]:
    """Residual add + LayerNorm in one pass, storing both h = x + residual and LN(h)."""
    _validate_fused_residual_layernorm_input(x, residual, weight, bias, eps)
    _validate_layernorm_output(x, out)
    _validate_layernorm_output(x, h_out)
    rows, cols = x.shape
    if rows == 0:
        return h_out, out
    _call("cuda_operator_fused_residual_layernorm_h", _ptr(x), _ptr(residual), _ptr(weight),
          _ptr(bias), _ptr(h_out), _ptr(out), int(rows), int(cols),
          float(eps), _stream(x))
    return h_out, out


def fused_residual_layernorm_h(x: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor,
                               bias: torch.Tensor,
                               eps: float = 1e-5) -> tuple[torch.Tensor, torch.Tensor]:
    """Allocating form of :func:`fused_residual_layernorm_h_into`; returns (h, y)."""
    return fused_residual_layernorm_h_into(x, residual, weight, bias, torch.empty_like(x),
                                           torch.empty_like(x), eps)


__all__ += ["fused_residual_layernorm_h_into", "fused_residual_layernorm_h"]

# ---------------------------------------------------------------- bias + GELU
# reference bindings.py:1394-1523


def _make_bias_gelu(version: int) -> None:
    symbol = f"cuda_operator_fused_bias_gelu_v{version}"

    def into(x: torch.Tensor, bias: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        if not x.is_cuda or not bias.is_cuda or not out.is_cuda:
            raise ValueError("fused bias GELU tensors must be CUDA tensors")
        if x.ndim != 2 or bias.ndim != 1 or bias.shape[0] != x.shape[1]:
            raise ValueError("expected x[rows, cols] and bias[cols]")
        if x.dtype != torch.float32 or bias.dtype != torch.float32 or out.dtype != torch.float32:
            raise TypeError("fused bias GELU currently supports float32 only")
        if out.shape != x.shape:
            raise ValueError("output shape must equal input shape")
        if not x.is_contiguous() or not bias.is_contiguous() or not out.is_contiguous():
            raise ValueError("all tensors must be contiguous")
        if x.shape[1] == 0:
            raise ValueError("cols must be > 0")
        rows, cols = x.shape
        if rows == 0:
            return out
        _call(symbol, _ptr(x), _ptr(bias), _ptr(out), int(rows),
              int(cols), _stream(x))
        return out

    def alloc(x: torch.Tensor, bias: torch.Tensor) -> torch.Tensor:
        return into(x, bias, torch.empty_like(x))

    doc = f"gelu_erf(x + bias[col]), fp32 (reference fused_bias_gelu_v{version})."
    _export(f"fused_bias_gelu_v{version}_into", into, doc)
    _export(f"fused_bias_gelu_v{version}", alloc, doc)


for _v in range(3):
    _make_bias_gelu(_v)

# ---------------------------------------------------------------- SwiGLU
# reference bindings.py:1526-1641


def _validate_swiglu(gate: torch.Tensor, up: torch.Tensor, out: torch.Tensor) -> None:
    if not gate.is_cuda or not up.is_cuda or not out.is_cuda:
        raise ValueError("SwiGLU tensors must be CUDA tensors")
    if gate.shape != up.shape or out.shape != gate.shape:
        raise ValueError("gate, up, and output must have the same shape")
    if gate.dtype != torch.float32 or up.dtype != torch.float32 or out.dtype != torch.float32:
        raise TypeError("SwiGLU currently supports float32 only")
    if not gate.is_contiguous() or not up.is_contiguous() or not out.is_contiguous():
        raise ValueError("SwiGLU tensors must be contiguous")


def _make_swiglu(version: int) -> None:
    symbol = f"cuda_operator_swiglu_v{version}"

    def into(gate: torch.Tensor, up: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        _validate_swiglu(gate, up, out)
        if version == 2:
            if gate.ndim != 2:
                raise ValueError("SwiGLU V2 expects a 2-D tensor")
            rows, cols = gate.shape
            if rows == 0:
                return out
            _call(symbol, _ptr(gate), _ptr(up), _ptr(out), int(rows),
                  int(cols), _stream(gate))
            return out
        if gate.numel() == 0:
            return out
        _call(symbol, _ptr(gate), _ptr(up), _ptr(out), int(gate.numel()),
              _stream(gate))
        return out

    def alloc(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
        return into(gate, up, torch.empty_like(gate))

    doc = f"silu(gate) * up, fp32 (reference swiglu_v{version})."
    _export(f"swiglu_v{version}_into", into, doc)
    _export(f"swiglu_v{version}", alloc, doc)


for _v in range(3):
    _make_swiglu(_v)

# ---------------------------------------------------------------- GEMM + bias + GELU
# reference bindings.py:1644-2033


def _make_gemm_bias_gelu(version: int) -> None:
    symbol = f"cuda_operator_gemm_bias_gelu_v{version}"

    def into(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor,
             out: torch.Tensor) -> torch.Tensor:
        if not _all_cuda(x, weight, bias, out):
            raise ValueError("GEMM Bias GELU tensors must be CUDA tensors")
        if x.ndim != 2 or weight.ndim != 2:
            raise ValueError("x and weight must be 2-D")
        if x.shape[1] != weight.shape[1]:
            raise ValueError("x.shape[1] must equal weight.shape[1]")
        if bias.ndim != 1 or bias.shape[0] != weight.shape[0]:
            raise ValueError("bias length must equal weight.shape[0]")
        expected_shape = (x.shape[0], weight.shape[0])
        if out.shape != expected_shape:
            raise ValueError(f"output shape must be {expected_shape}")
        if _any_not_dtype(torch.float32, x, weight, bias, out):
            raise TypeError("GEMM Bias GELU currently supports float32 only")
        if not _all_contiguous(x, weight, bias, out):
            raise ValueError("all GEMM Bias GELU tensors must be contiguous")
        m, k = x.shape
        n = weight.shape[0]
        if m == 0 or n == 0:
            return out
        _call(symbol, _ptr(x), _ptr(weight), _ptr(bias), _ptr(out), int(m),
              int(k), int(n), _stream(x))
        return out

    def alloc(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor) -> torch.Tensor:
        out = torch.empty((x.shape[0], weight.shape[0]), device=x.device, dtype=torch.float32)
        return into(x, weight, bias, out)

    form = "erf" if version <= 1 else "tanh"
    doc = f"gelu_{form}(x @ weight.T + bias), fp32 (reference gemm_bias_gelu_v{version})."
    _export(f"gemm_bias_gelu_v{version}_into", into, doc)
    _export(f"gemm_bias_gelu_v{version}", alloc, doc)


for _v in range(7):
    _make_gemm_bias_gelu(_v)


def gemm_bias_gelu_bf16_into(x_bf16: torch.Tensor, weight_bf16: torch.Tensor, bias: torch.Tensor,
                             out_bf16: torch.Tensor) -> torch.Tensor:
    """bf16 tensor-core gelu_erf(x @ W.T + bias) with fp32 accumulation and bf16 output."""
    if not _all_cuda(x_bf16, weight_bf16, bias, out_bf16):
        raise ValueError("GEMM Bias GELU tensors must be CUDA tensors")
    if x_bf16.ndim != 2 or weight_bf16.ndim != 2:
        raise ValueError("x and weight must be 2-D")
    if x_bf16.shape[1] != weight_bf16.shape[1]:
        raise ValueError("x.shape[1] must equal weight.shape[1]")
    if bias.ndim != 1 or bias.shape[0] != weight_bf16.shape[0]:
        raise ValueError("bias length must equal weight.shape[0]")
    expected_shape = (x_bf16.shape[0], weight_bf16.shape[0])
    if out_bf16.shape != expected_shape:
        raise ValueError(f"output shape must be {expected_shape}")
    if _any_not_dtype(torch.bfloat16, x_bf16, weight_bf16, out_bf16):
        raise TypeError("GEMM Bias GELU bf16 expects bfloat16 x, weight and output")
    if bias.dtype != torch.float32:
        raise TypeError("GEMM Bias GELU bf16 expects a float32 bias")
    if not _all_contiguous(x_bf16, weight_bf16, bias, out_bf16):
        raise ValueError("all GEMM Bias GELU tensors must be contiguous")
    m, k = x_bf16.shape
    n = weight_bf16.shape[0]
    if m == 0 or n == 0:
        return out_bf16
    _call("cuda_operator_gemm_bias_gelu_bf16", _ptr(x_bf16), _ptr(weight_bf16), _ptr(bias),
          _ptr(out_bf16), int(m), int(k), int(n),
          _stream(x_bf16))
    return out_bf16


def gemm_bias_gelu_bf16(x_bf16: torch.Tensor, weight_bf16: torch.Tensor,
                        bias: torch.Tensor) -> torch.Tensor:
    """Allocating form of :func:`gemm_bias_gelu_bf16_into`."""
    out = torch.empty((x_bf16.shape[0], weight_bf16.shape[0]), device=x_bf16.device,
                      dtype=torch.bfloat16)
    return gemm_bias_gelu_bf16_into(x_bf16, weight_bf16, bias, out)


__all__ += ["gemm_bias_gelu_bf16_into", "gemm_bias_gelu_bf16"]


def gemm_residual_bf16_into(x_bf16: torch.Tensor, weight_bf16: torch.Tensor,
                            residual_bf16: torch.Tensor, out_bf16: torch.Tensor) -> torch.Tensor:
    """Down projection with the residual add fused: out = bf16(x @ W.T + residual).

    bf16 x [M, K], W [N, K], residual and out [M, N]; fp32 accumulation.
    ``out_bf16`` may be ``residual_bf16`` itself (in-place residual update).
    """
    tensors = (x_bf16, weight_bf16, residual_bf16, out_bf16)
    if not _all_cuda(*tensors):
        raise ValueError("GEMM residual tensors must be CUDA tensors")
    if x_bf16.ndim != 2 or weight_bf16.ndim != 2:
        raise ValueError("x and weight must be 2-D")
    if x_bf16.shape[1] != weight_bf16.shape[1]:
        raise ValueError("x.shape[1] must equal weight.shape[1]")
    expected_shape = (x_bf16.shape[0], weight_bf16.shape[0])
    if residual_bf16.shape != expected_shape or out_bf16.shape != expected_shape:
        raise ValueError(f"residual and output shape must be {expected_shape}")
    if _any_not_dtype(torch.bfloat16, *tensors):
        raise TypeError("GEMM residual bf16 expects bfloat16 tensors")
    if not _all_contiguous(*tensors):
        raise ValueError("all GEMM residual tensors must be contiguous")
    m, k = x_bf16.shape
    n = weight_bf16.shape[0]
    if m == 0 or n == 0:
        return out_bf16
    if k == 0:
        raise ValueError("GEMM residual requires k > 0")
    _call("cuda_operator_gemm_residual_bf16", _ptr(x_bf16), _ptr(weight_bf16),
          _ptr(residual_bf16), _ptr(out_bf16), int(m), int(k),
          int(n), _stream(x_bf16))
    return out_bf16


def gemm_residual_bf16(x_bf16: torch.Tensor, weight_bf16: torch.Tensor,
                       residual_bf16: torch.Tensor) -> torch.Tensor:
    """Allocating form of :func:`gemm_residual_bf16_into`."""
    out = torch.empty((x_bf16.shape[0], weight_bf16.shape[0]), device=x_bf16.device,
                      dtype=torch.bfloat16)
    return gemm_residual_bf16_into(x_bf16, weight_bf16, residual_bf16, out)


__all__ += ["gemm_residual_bf16_into", "gemm_residual_bf16"]

# ---------------------------------------------------------------- RMSNorm folded into the GEMM


def rmsnorm_rstd_bf16_into(x_bf16: torch.Tensor, rstd: torch.Tensor,
                           eps: float = 1e-5) -> torch.Tensor:
    """Per-row inverse RMS of bf16 x: rstd[row] = rsqrt(mean(x[row]^2) + eps), fp32."""
    if not x_bf16.is_cuda or not rstd.is_cuda:
        raise ValueError("rmsnorm input and rstd must be CUDA tensors")
    if x_bf16.ndim != 2 or x_bf16.dtype != torch.bfloat16 or not x_bf16.is_contiguous():
        raise ValueError("rmsnorm_rstd_bf16 expects a contiguous 2-D bfloat16 input")
    if rstd.shape != (x_bf16.shape[0],) or rstd.dtype != torch.float32 or not rstd.is_contiguous():
        raise ValueError("rstd must be a contiguous float32 vector of length rows")
    if x_bf16.shape[1] == 0:
        raise ValueError("rmsnorm requires cols > 0")
    if eps <= 0:
        raise ValueError("rmsnorm eps must be positive")
    rows, cols = x_bf16.shape
    if rows == 0:
        return rstd
    _call("cuda_operator_rmsnorm_rstd_bf16", _ptr(x_bf16), _ptr(rstd), int(rows),
          int(cols), float(eps), _stream(x_bf16))
    return rstd


def rmsnorm_rstd_bf16(x_bf16: torch.Tensor, eps: float = 1e-5) -> torch.Tensor:
    """Allocating form of :func:`rmsnorm_rstd_bf16_into`."""
    return rmsnorm_rstd_bf16_into(
        x_bf16, torch.empty(x_bf16.shape[0], device=x_bf16.device, dtype=torch.float32), eps)


def fold_rmsnorm_weight(packed_weight_bf16: torch.Tensor,
                        norm_weight_bf16: torch.Tensor) -> torch.Tensor:
    """W * diag(w) for :func:`gemm_swiglu_rowscale_bf16`: every column k of the packed
    [2N, K] weight multiplied by the RMSNorm weight w[k] (fp32 product, rounded once
    to bf16).  A one-time weight transform, like packing."""
    if packed_weight_bf16.ndim != 2 or norm_weight_bf16.shape != (packed_weight_bf16.shape[1],):
        raise ValueError("norm weight length must equal the packed weight's K")
    return (packed_weight_bf16.float() * norm_weight_bf16.float()[None, :]).to(torch.bfloat16)


def gemm_swiglu_rowscale_bf16_into(x_bf16: torch.Tensor, row_scale: torch.Tensor,
                                   packed_weight_bf16: torch.Tensor,
                                   out_bf16: torch.Tensor) -> torch.Tensor:
    """bf16(silu(rs * (x @ Wg.T)) * (rs * (x @ Wu.T))) with rs = row_scale[row]: the
    RMSNorm -> GEMM+SwiGLU block when the weight was folded by :func:`fold_rmsnorm_weight`
    and row_scale comes from :func:`rmsnorm_rstd_bf16`."""
    tensors = (x_bf16, row_scale, packed_weight_bf16, out_bf16)
    if not _all_cuda(*tensors):
        raise ValueError("GEMM SwiGLU tensors must be CUDA tensors")
    if x_bf16.ndim != 2 or packed_weight_bf16.ndim != 2:
        raise ValueError("x and packed weight must be 2-D")
    if x_bf16.shape[1] != packed_weight_bf16.shape[1] or packed_weight_bf16.shape[0] % 2:
        raise ValueError("packed weight must be [2N, K] with K = x.shape[1]")
    n = packed_weight_bf16.shape[0] // 2
    m, k = x_bf16.shape
    if row_scale.shape != (m,) or row_scale.dtype != torch.float32:
        raise ValueError("row_scale must be a float32 vector of length M")
    if out_bf16.shape != (m, n):
        raise ValueError(f"output shape must be {(m, n)}")
    if _any_not_dtype(torch.bfloat16, x_bf16, packed_weight_bf16, out_bf16):
        raise TypeError("GEMM SwiGLU row-scale expects bfloat16 x, weight and output")
    if not _all_contiguous(*tensors):
        raise ValueError("all GEMM SwiGLU tensors must be contiguous")
    if m == 0 or n == 0:
        return out_bf16
    _call("cuda_operator_gemm_swiglu_rowscale_bf16", _ptr(x_bf16), _ptr(row_scale),
          _ptr(packed_weight_bf16), _ptr(out_bf16), int(m), int(k),
          int(n), _stream(x_bf16))
    return out_bf16


def gemm_swiglu_rowscale_bf16(x_bf16: torch.Tensor, row_scale: torch.Tensor,
                              packed_weight_bf16: torch.Tensor) -> torch.Tensor:
    """Allocating form of :func:`gemm_swiglu_rowscale_bf16_into`."""
    out = torch.empty((x_bf16.shape[0], packed_weight_bf16.shape[0] // 2), device=x_bf16.device,
                      dtype=torch.bfloat16)
    return gemm_swiglu_rowscale_bf16_into(x_bf16, row_scale, packed_weight_bf16, out)


__all__ += ["rmsnorm_rstd_bf16_into", "rmsnorm_rstd_bf16", "fold_rmsnorm_weight",
            "gemm_swiglu_rowscale_bf16_into", "gemm_swiglu_rowscale_bf16"]

# ---------------------------------------------------------------- GEMM + SwiGLU + all-gather
# no reference counterpart: the N-sharded GEMM whose epilogue also stores its
# output block into the other ranks' outputs (peer memory over NVLink)


def gemm_swiglu_allgather_bf16(x_bf16: torch.Tensor, row_scale: torch.Tensor | None,
                               packed_weight_bf16: torch.Tensor, dests: Sequence[int],
                               ld: int) -> None:
    """bf16(silu(rs * g) * (rs * u)) of this rank's packed weight shard [2n, K]
    (rs = row_scale[row], or 1 when row_scale is None), stored to every address in
    ``dests``: each is the origin of this rank's [M, n] column block inside an
    [M, ld] bf16 output -- this GPU's own first, then the other ranks' as mapped by
    :func:`peer_open`.  Enqueued on the current stream of x's device; follow it
    with :func:`peer_barrier` before reading blocks other ranks wrote."""
    tensors = [x_bf16, packed_weight_bf16] + ([row_scale] if row_scale is not None else [])
    if not _all_cuda(*tensors):
        raise ValueError("GEMM SwiGLU tensors must be CUDA tensors")
    if x_bf16.ndim != 2 or packed_weight_bf16.ndim != 2:
        raise ValueError("x and packed weight must be 2-D")
    if x_bf16.shape[1] != packed_weight_bf16.shape[1] or packed_weight_bf16.shape[0] % 2:
        raise ValueError("packed weight must be [2N, K] with K = x.shape[1]")
    if x_bf16.dtype != torch.bfloat16 or packed_weight_bf16.dtype != torch.bfloat16:
        raise TypeError("GEMM SwiGLU all-gather expects bfloat16 x and weight")
    if not _all_contiguous(*tensors):
        raise ValueError("all GEMM SwiGLU tensors must be contiguous")
    n = packed_weight_bf16.shape[0] // 2
    m, k = x_bf16.shape
    if row_scale is not None and (row_scale.shape != (m,) or row_scale.dtype != torch.float32):
        raise ValueError("row_scale must be a float32 vector of length M")
    if not 1 <= len(dests) <= 8 or any(int(d) == 0 for d in dests):
        raise ValueError("dests must hold 1 to 8 non-null device addresses")
    if ld < n:
        raise ValueError("ld must be at least the block width n")
    if m == 0 or n == 0:
        return
    array = (ctypes.c_void_p * len(dests))(*[int(d) for d in dests])
    _call("cuda_operator_gemm_swiglu_allgather_bf16", _ptr(x_bf16),
          _ptr(row_scale) if row_scale is not None else None,
          _ptr(packed_weight_bf16), array, int(len(dests)), int(m),
          int(k), int(n), int(ld), _stream(x_bf16))


def rmsnorm_allgather_bf16(x_bf16: torch.Tensor, weight_bf16: torch.Tensor,
                           dests: Sequence[int], eps: float = 1e-5) -> None:
    """bf16 RMSNorm of x [rows, cols] (bit for bit :func:`rmsnorm_bf16`) stored
    to every address in ``dests``: each is where these rows go in a bf16
    buffer with row stride cols -- this GPU's first, then the other ranks' as
    mapped by :func:`peer_open`.  Enqueued on the current stream of x's device;
    follow it with :func:`peer_barrier` before other ranks read the rows.
    cols must be a multiple of 8 and at most 8192."""
    if not _all_cuda(x_bf16, weight_bf16):
        raise ValueError("RMSNorm tensors must be CUDA tensors")
    if x_bf16.ndim != 2 or weight_bf16.ndim != 1 or weight_bf16.shape[0] != x_bf16.shape[1]:
        raise ValueError("expected x [rows, cols] and a weight of cols elements")
    if x_bf16.dtype != torch.bfloat16 or weight_bf16.dtype != torch.bfloat16:
        raise TypeError("RMSNorm all-gather expects bfloat16 x and weight")
    if not _all_contiguous(x_bf16, weight_bf16):
        raise ValueError("RMSNorm tensors must be contiguous")
    if x_bf16.shape[1] % 8 or x_bf16.shape[1] > 8192:
        raise ValueError("cols must be a multiple of 8 and at most 8192")
    if not 1 <= len(dests) <= 8 or any(int(d) == 0 for d in dests):
        raise ValueError("dests must hold 1 to 8 non-null device addresses")
    if eps <= 0:
        raise ValueError("eps must be positive")
    rows, cols = x_bf16.shape
    if rows == 0:
        return
    array = (ctypes.c_void_p * len(dests))(*[int(d) for d in dests])
    _call("cuda_operator_rmsnorm_allgather_bf16", _ptr(x_bf16), _ptr(weight_bf16), array,
          int(len(dests)), int(rows), int(cols), float(eps), _stream(x_bf16))


def peer_alloc(nbytes: int) -> tuple[int, bytes]:
    """Zero-filled device allocation on the current device that other processes
    can map: (address, handle bytes to send them)."""
    library = _library()
    size = int(library.handle.cuda_operator_lab_peer_handle_bytes())
    handle = ctypes.create_string_buffer(size)
    addr = ctypes.c_void_p()
    library.check(library.handle.cuda_operator_lab_peer_alloc(
        int(nbytes), ctypes.byref(addr), handle))
    return int(addr.value), handle.raw


def peer_open(handle: bytes) -> int:
    """Address of another process's :func:`peer_alloc` allocation in this process."""
    addr = ctypes.c_void_p()
    buf = ctypes.create_string_buffer(bytes(handle), len(handle))
    _call("cuda_operator_lab_peer_open", buf, ctypes.byref(addr))
    return int(addr.value)


def peer_close(addr: int) -> None:
    """Unmaps an address returned by :func:`peer_open`."""
    _call("cuda_operator_lab_peer_close", ctypes.c_void_p(addr))


def peer_free(addr: int) -> None:
    """Frees a :func:`peer_alloc` allocation (after every peer closed its mapping)."""
    _call("cuda_operator_lab_peer_free", ctypes.c_void_p(addr))


def peer_barrier(flag_addrs: Sequence[int], rank: int, epoch: int,
                 timeout_ns: int = 5_000_000_000, stream: torch.cuda.Stream | None = None) -> None:
    """Enqueues the device-side barrier of len(flag_addrs) ranks at ``epoch`` on
    ``stream`` (default: the current stream).  flag_addrs[j] is rank j's
    zero-initialised uint32 flag array as mapped here; epochs increase per call.  A
    wait longer than timeout_ns sets the :func:`peer_status` bit instead of hanging."""
    world = len(flag_addrs)
    if not 1 <= world <= 8 or not 0 <= rank < world:
        raise ValueError("need 1 <= world <= 8 and 0 <= rank < world")
    array = (ctypes.c_void_p * world)(*[int(a) for a in flag_addrs])
    s = stream if stream is not None else torch.cuda.current_stream()
    _call("cuda_operator_lab_peer_barrier", array, int(rank), int(world),
          int(epoch & 0xFFFFFFFF), int(timeout_ns),
          ctypes.c_void_p(s.cuda_stream))


def peer_status(clear: bool = True) -> int:
    """Peer status word of the current device (bit 1: a barrier wait timed out).
    Synchronises the device."""
    value = ctypes.c_uint(0)
    _call("cuda_operator_lab_peer_status", ctypes.byref(value), int(1 if clear else 0))
    return int(value.value)


__all__ += ["gemm_swiglu_allgather_bf16", "rmsnorm_allgather_bf16", "peer_alloc", "peer_open", "peer_close", "peer_free",
            "peer_barrier", "peer_status"]

# ---------------------------------------------------------------- GEMM + SwiGLU
# reference bindings.py:2036-2818


def _make_gemm_swiglu_f32_dual(version: int) -> None:
    """v0/v1: fp32 X, separate gate/up weights, fp32 workspace and output."""
    symbol = f"cuda_operator_gemm_swiglu_v{version}"

    def into(x: torch.Tensor, gate_weight: torch.Tensor, up_weight: torch.Tensor,
             workspace: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        if not _all_cuda(x, gate_weight, up_weight, workspace, out):
            raise ValueError("GEMM SwiGLU tensors must be CUDA tensors")
        if x.ndim != 2 or gate_weight.ndim != 2 or up_weight.ndim != 2:
            raise ValueError("x and weights must be 2-D")
        if gate_weight.shape != up_weight.shape:
            raise ValueError("gate_weight and up_weight must have the same shape")
        if x.shape[1] != gate_weight.shape[1]:
            raise ValueError("x.shape[1] must equal weight.shape[1]")
        expected_shape = (x.shape[0], gate_weight.shape[0])
        if workspace.shape != expected_shape or out.shape != expected_shape:
            raise ValueError(f"workspace and output shape must be {expected_shape}")
        if _any_not_dtype(torch.float32, x, gate_weight, up_weight, workspace, out):
            raise TypeError("GEMM SwiGLU currently supports float32 only")
        if not _all_contiguous(x, gate_weight, up_weight, workspace, out):
            raise ValueError("all GEMM SwiGLU tensors must be contiguous")
        m, k = x.shape
        n = gate_weight.shape[0]
        if m == 0 or n == 0:
            return out
        if workspace.data_ptr() == out.data_ptr():
            raise ValueError("workspace and output must not alias")
        _call(symbol, _ptr(x), _ptr(gate_weight), _ptr(up_weight), _ptr(workspace), _ptr(out),
              int(m), int(k), int(n), _stream(x))
        return out

    def alloc(x: torch.Tensor, gate_weight: torch.Tensor, up_weight: torch.Tensor) -> torch.Tensor:
        shape = (x.shape[0], gate_weight.shape[0])
        workspace = torch.empty(shape, device=x.device, dtype=torch.float32)
        out = torch.empty(shape, device=x.device, dtype=torch.float32)
        return into(x, gate_weight, up_weight, workspace, out)

    doc = f"silu(x @ Wg.T) * (x @ Wu.T), fp32 (reference gemm_swiglu_v{version})."
    _export(f"gemm_swiglu_v{version}_into", into, doc)
    _export(f"gemm_swiglu_v{version}", alloc, doc)


def _make_gemm_swiglu_packed(version: int, in_dtype: torch.dtype, ws_dtype: torch.dtype,
                             doc: str) -> None:
    """v2/v3 (fp32), v4/v10/v11 (bf16, fp32 workspace), v5 (bf16 workspace)."""
    symbol = f"cuda_operator_gemm_swiglu_v{version}"
    tag = f"V{version}"
    bf16 = in_dtype == torch.bfloat16

    def into(x: torch.Tensor, packed_weight: torch.Tensor, workspace: torch.Tensor,
             out: torch.Tensor) -> torch.Tensor:
        # Fast path: every check below in one expression, each attribute read
        # once (a small GEMM's call is host-bound).  Anything it rejects goes
        # through the checks in the reference's order for the exact error.
        xs, ps = x.shape, packed_weight.shape
        if (len(xs) == 2 and len(ps) == 2 and xs[1] == ps[1] and not ps[0] & 1
                and x.dtype is in_dtype and packed_weight.dtype is in_dtype
                and workspace.dtype is ws_dtype and out.dtype is torch.float32
                and x.is_cuda and packed_weight.is_cuda and workspace.is_cuda and out.is_cuda
                and workspace.shape == (xs[0], ps[0]) and out.shape == (xs[0], ps[0] >> 1)
                and x.is_contiguous() and packed_weight.is_contiguous()
                and workspace.is_contiguous() and out.is_contiguous()):
            if xs[0] and ps[0]:
                _call(symbol, x.data_ptr(), packed_weight.data_ptr(), workspace.data_ptr(),
                      out.data_ptr(), xs[0], xs[1], ps[0] >> 1, _stream(x))
            return out
        return checked_into(x, packed_weight, workspace, out)

    def checked_into(x: torch.Tensor, packed_weight: torch.Tensor, workspace: torch.Tensor,
                     out: torch.Tensor) -> torch.Tensor:
        if not _all_cuda(x, packed_weight, workspace, out):
            raise ValueError(f"GEMM SwiGLU {tag} tensors must be CUDA tensors")
        if x.ndim != 2 or packed_weight.ndim != 2:
            raise ValueError("x_bf16 and packed_weight_bf16 must be 2-D" if bf16
                             else "x and packed_weight must be 2-D")
        if x.shape[1] != packed_weight.shape[1]:
            if version in (4, 5):
                raise ValueError("x_bf16.shape[1] must equal packed_weight_bf16.shape[1]")
            if version in (10, 11):
                raise ValueError("x.shape[1] must equal packed_weight.shape[1]")
            raise ValueError("x.shape[1] must equal packed_weight.shape[1]")
        if packed_weight.shape[0] % 2 != 0:
            raise ValueError("packed_weight_bf16.shape[0] must be even" if version in (4, 5)
                             else "packed_weight.shape[0] must be even")
        if bf16:
            if x.dtype != torch.bfloat16 or packed_weight.dtype != torch.bfloat16:
                raise TypeError(f"GEMM SwiGLU {tag} expects BF16 input and packed weight")
            if version == 5:
                if workspace.dtype != torch.bfloat16:
                    raise TypeError("GEMM SwiGLU V5 workspace must be BF16")
                if out.dtype != torch.float32:
                    raise TypeError("GEMM SwiGLU V5 output must be float32")
            elif workspace.dtype != torch.float32 or out.dtype != torch.float32:
                if version == 4:
                    raise TypeError("GEMM SwiGLU V4 workspace and output must be float32")
                raise TypeError(f"GEMM SwiGLU {tag} workspace/output must be float32")
        n = packed_weight.shape[0] // 2
        expected_workspace = (x.shape[0], 2 * n)
        expected_out = (x.shape[0], n)
        if workspace.shape != expected_workspace:
            raise ValueError(f"workspace shape must be {expected_workspace}")
        if out.shape != expected_out:
            raise ValueError(f"output shape must be {expected_out}")
        if not bf16 and _any_not_dtype(torch.float32, x, packed_weight, workspace, out):
            raise TypeError(f"GEMM SwiGLU {tag} currently supports float32 only")
        if not _all_contiguous(x, packed_weight, workspace, out):
            raise ValueError(f"all GEMM SwiGLU {tag} tensors must be contiguous")
        m, k = x.shape
        if m == 0 or n == 0:
            return out
        _call(symbol, _ptr(x), _ptr(packed_weight), _ptr(workspace), _ptr(out),
              int(m), int(k), int(n), _stream(x))
        return out

    def alloc(x: torch.Tensor, packed_weight: torch.Tensor) -> torch.Tensor:
        n = packed_weight.shape[0] // 2
        workspace = torch.empty((x.shape[0], 2 * n), device=x.device, dtype=ws_dtype)
        out = torch.empty((x.shape[0], n), device=x.device, dtype=torch.float32)
        return into(x, packed_weight, workspace, out)

    _export(f"gemm_swiglu_v{version}_into", into, doc)
    _export(f"gemm_swiglu_v{version}", alloc, doc)


_BF16_DUAL_GUARDS = {
    6: ((16, 16, 16), "GEMM SwiGLU V6 requires M, K, and N to be multiples of 16"),
    7: ((16, 16, 64), "GEMM SwiGLU V7 requires M and K multiples of 16 and N multiple of 64"),
    8: ((32, 16, 64),
        "GEMM SwiGLU V8 requires M multiple of 32, K multiple of 16, and N multiple of 64"),
    9: ((16, 16, 128), "GEMM SwiGLU V9 requires M,K multiples of 16 and N multiple of 128"),
}


def _make_gemm_swiglu_bf16_dual(version: int) -> None:
    """v6..v9: bf16 X, separate bf16 gate/up weights, fp32 output, shape guards."""
    symbol = f"cuda_operator_gemm_swiglu_v{version}"
    tag = f"V{version}"
    (m_mult, k_mult, n_mult), guard_message = _BF16_DUAL_GUARDS[version]

    def into(x_bf16: torch.Tensor, gate_weight_bf16: torch.Tensor, up_weight_bf16: torch.Tensor,
             out: torch.Tensor) -> torch.Tensor:
        tensors = (x_bf16, gate_weight_bf16, up_weight_bf16, out)
        if not _all_cuda(*tensors):
            raise ValueError(f"GEMM SwiGLU {tag} tensors must be CUDA tensors")
        if x_bf16.ndim != 2 or gate_weight_bf16.ndim != 2 or up_weight_bf16.ndim != 2:
            raise ValueError("x and weights must be 2-D")
        if gate_weight_bf16.shape != up_weight_bf16.shape:
            raise ValueError("gate and up weights must have the same shape")
        if x_bf16.shape[1] != gate_weight_bf16.shape[1]:
            raise ValueError("x.shape[1] must equal weight.shape[1]")
        if _any_not_dtype(torch.bfloat16, x_bf16, gate_weight_bf16, up_weight_bf16):
            raise TypeError(f"GEMM SwiGLU {tag} expects BF16 input and weights")
        if out.dtype != torch.float32:
            raise TypeError(f"GEMM SwiGLU {tag} output must be float32")
        expected_out = (x_bf16.shape[0], gate_weight_bf16.shape[0])
        if out.shape != expected_out:
            raise ValueError(f"output shape must be {expected_out}")
        if not _all_contiguous(*tensors):
            raise ValueError(f"all GEMM SwiGLU {tag} tensors must be contiguous")
        m, k = x_bf16.shape
        n = gate_weight_bf16.shape[0]
        if m == 0 or n == 0:
            return out
        if (m % m_mult) != 0 or (k % k_mult) != 0 or (n % n_mult) != 0:
            raise ValueError(guard_message)
        _call(symbol, _ptr(x_bf16), _ptr(gate_weight_bf16), _ptr(up_weight_bf16), _ptr(out),
              int(m), int(k), int(n), _stream(x_bf16))
        return out

    def alloc(x_bf16: torch.Tensor, gate_weight_bf16: torch.Tensor,
              up_weight_bf16: torch.Tensor) -> torch.Tensor:
        out = torch.empty((x_bf16.shape[0], gate_weight_bf16.shape[0]), device=x_bf16.device,
                          dtype=torch.float32)
        return into(x_bf16, gate_weight_bf16, up_weight_bf16, out)

    doc = (f"silu(x @ Wg.T) * (x @ Wu.T) from bf16 operands, fp32 accumulate and output "
           f"(reference gemm_swiglu_v{version}).")
    _export(f"gemm_swiglu_v{version}_into", into, doc)
    _export(f"gemm_swiglu_v{version}", alloc, doc)


for _v in (0, 1):
    _make_gemm_swiglu_f32_dual(_v)
for _v in (2, 3):
    _make_gemm_swiglu_packed(_v, torch.float32, torch.float32,
                             f"Packed fp32 GEMM+SwiGLU (reference gemm_swiglu_v{_v}).")
for _v in (4, 10, 11):
    _make_gemm_swiglu_packed(
        _v, torch.bfloat16, torch.float32,
        f"Packed bf16 GEMM+SwiGLU on tcgen05 tensor cores, fp32 accumulate and output "
        f"(reference gemm_swiglu_v{_v}); the workspace is validated but not used.")
_make_gemm_swiglu_packed(
    5, torch.bfloat16, torch.bfloat16,
    "Packed bf16 GEMM+SwiGLU whose gate/up projections are rounded to bf16 before SiLU "
    "(reference gemm_swiglu_v5); the workspace is validated but not used.")
for _v in (6, 7, 8, 9):
    _make_gemm_swiglu_bf16_dual(_v)


def gemm_swiglu_bf16_into(x_bf16: torch.Tensor, packed_weight_bf16: torch.Tensor,
                          out_bf16: torch.Tensor) -> torch.Tensor:
    """Packed bf16 GEMM+SwiGLU with bf16 output: bf16(silu(x@Wg.T) * (x@Wu.T)).

    packed_weight_bf16 is [2N, K] with the N gate rows first.  No workspace:
    both projections stay in tensor memory until the fused epilogue.
    """
    tensors = (x_bf16, packed_weight_bf16, out_bf16)
    if not _all_cuda(*tensors):
        raise ValueError("GEMM SwiGLU bf16 tensors must be CUDA tensors")
    if x_bf16.ndim != 2 or packed_weight_bf16.ndim != 2:
        raise ValueError("x_bf16 and packed_weight_bf16 must be 2-D")
    if x_bf16.shape[1] != packed_weight_bf16.shape[1]:
        raise ValueError("x_bf16.shape[1] must equal packed_weight_bf16.shape[1]")
    if packed_weight_bf16.shape[0] % 2 != 0:
        raise ValueError("packed_weight_bf16.shape[0] must be even")
    if _any_not_dtype(torch.bfloat16, *tensors):
        raise TypeError("GEMM SwiGLU bf16 expects bfloat16 input, packed weight and output")
    n = packed_weight_bf16.shape[0] // 2
    expected_out = (x_bf16.shape[0], n)
    if out_bf16.shape != expected_out:
        raise ValueError(f"output shape must be {expected_out}")
    if not _all_contiguous(*tensors):
        raise ValueError("all GEMM SwiGLU bf16 tensors must be contiguous")
    m, k = x_bf16.shape
    if m == 0 or n == 0:
        return out_bf16
    _call("cuda_operator_gemm_swiglu_bf16", _ptr(x_bf16), _ptr(packed_weight_bf16), _ptr(out_bf16),
          int(m), int(k), int(n), _stream(x_bf16))
    return out_bf16


def gemm_swiglu_bf16(x_bf16: torch.Tensor, packed_weight_bf16: torch.Tensor) -> torch.Tensor:
    """Allocating form of :func:`gemm_swiglu_bf16_into`."""
    out = torch.empty((x_bf16.shape[0], packed_weight_bf16.shape[0] // 2), device=x_bf16.device,
                      dtype=torch.bfloat16)
    return gemm_swiglu_bf16_into(x_bf16, packed_weight_bf16, out)


__all__ += ["gemm_swiglu_bf16_into", "gemm_swiglu_bf16"]

# ---------------------------------------------------------------- library info


def gemm_status(clear: bool = True) -> int:
    """Bounded-wait status word of the tensor-core GEMM on the current device.

    0 means no mbarrier wait ever ran out of time.  Synchronises the device.
    """
    value = ctypes.c_uint(0)
    _call("cuda_operator_lab_gemm_status", ctypes.byref(value), int(1 if clear else 0))
    return int(value.value)


def device_info() -> dict[str, int]:
    """SM count and compute capability of the current device, as the library sees them."""
    sm, major, minor = ctypes.c_int(0), ctypes.c_int(0), ctypes.c_int(0)
    _call("cuda_operator_lab_device_info", ctypes.byref(sm), ctypes.byref(major),
          ctypes.byref(minor))
    return {"sm_count": sm.value, "cc_major": major.value, "cc_minor": minor.value}


def build_tag() -> str:
    """Build tag string compiled into the loaded library."""
    return _library().handle.cuda_operator_lab_build_tag().decode()


__all__ += ["gemm_status", "device_info", "build_tag", "library_path", "REFERENCE_SYMBOLS"]
