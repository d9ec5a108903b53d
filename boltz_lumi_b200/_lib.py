"""ctypes binding of ``libboltz_b200.so`` (the C ABI of ``include/boltz_b200.h``).

The library is loaded once, from the package directory.  If it is missing the
import of any op fails loudly: there is no CPU or eager fallback for the
kernels.  Every call passes raw device pointers and the current CUDA stream
and turns a non-zero status into ``RuntimeError`` carrying ``bl_last_error()``.
"""

import ctypes
from ctypes import c_float, c_int, c_int64, c_void_p
from pathlib import Path

import torch

LIBRARY_PATH = Path(__file__).resolve().parent / "libboltz_b200.so"

BL_F32, BL_BF16 = 0, 1
BL_EPI_MODULATION, BL_EPI_GATE, BL_EPI_GATED_SWIGLU, BL_EPI_SWIGLU = 0, 1, 3, 2

_p = c_void_p
_i64p = ctypes.POINTER(c_int64)

# name -> argument types (restype is int unless listed in _RESTYPES)
SIGNATURES = {
    "bl_last_error": [],
    "bl_version": [],
    "bl_device_status": [c_int],
    "bl_wait_selftest": [c_int, c_int64, _p],
    "bl_layernorm": [_p, c_int, c_int64, c_int64, c_int, _p, _p, c_float, _p, c_int, _p],
    "bl_gate": [_p, _p, _p, c_int64, _p],
    "bl_gate_pack": [_p, _p, c_int64, _p, c_int64, c_int, _p, _p, _p],
    "bl_gate_split": [_p, _p, c_int64, _p, c_int64, _p, _p, _p],
    "bl_silu_mul": [_p, _p, _p, c_int64, _p],
    "bl_diffusion_epilogue": [_p, _p, _p, _p, c_int64, c_int64, c_int, _p],
    "bl_adaln_modulate": [_p, _p, _p, _p, c_int64, c_int64, c_float, _p],
    "bl_triangle_softmax": [_p, c_int, c_int64, c_int64, c_int64, c_int64, _i64p, _p, _i64p, _p, _i64p, _p, _p],
    "bl_batched_gemm": [_p, c_int, c_int64, c_int64, _p, c_int, c_int64, c_int64, _p, c_int64, c_int64,
                        c_int64, c_int64, c_int64, c_int64, _p, _p],
    "bl_linear_fused": [_p, c_int64, _p, c_int64, c_int64, _p, c_int64, c_int64, c_int64, c_int64, _p, c_int, _p,
                        c_int64, _p, c_int64, _p],
    "bl_attention_projection": [_p, c_int64, c_int64, _p, _p, c_float, _p, _p, c_float, _p, c_int, _p, c_int64, _p,
                                c_int64, c_int64, _p],
    "bl_trimul_projection": [_p, c_int64, c_int64, _p, _p, c_float, _p, _p, _p, c_int64, _p, _p],
    "bl_pair_transition": [_p, c_int64, _p, _p, c_float, _p, _p, _p, _p, _p],
    "bl_trimul_output": [_p, c_int64, c_int64, c_int64, _p, _p, c_float, _p, _p, _p, _p, _p],
    "bl_pair_bias": [_p, c_int64, _p, _p, c_float, _p, c_int64, _p, _p],
    "bl_swiglu_rows": [_p, c_int64, c_int64, c_int64, _p, c_int64, _p],
    "bl_triangle_attention": [_p, _p, _p, _p, c_int64, c_int64, c_int64, _p, c_int64, c_int64, _p, c_int64,
                              c_int64, c_float, c_int64, c_int64, c_int64, c_int64, _p, c_int64, _p],
    "bl_triangle_attention_residual": [_p, _p, _p, _p, c_int64, c_int64, c_int64, _p, c_int64, c_int64, _p, c_int64,
                                       c_int64, c_float, c_int64, c_int64, c_int64, c_int64, _p, c_int64, _p, _p, _p,
                                       c_int64, _p],
    "bl_pair_transition_static": [_p, c_int64, _p, _p, c_float, _p, _p, _p, _p],
    "bl_split3_bf16": [_p, c_int64, c_int64, c_int64, _p, _p],
    "bl_linear_split3": [_p, c_int64, c_int64, _p, c_int64, _p, _p, c_int64, _p, c_int64, _p],
    "bl_token_attention": [_p, _p, _p, _p, c_int64, c_int64, c_int64, _p, c_int64, c_int64, c_int64, c_int64, c_int64,
                           _p, c_int64, c_float, c_float, c_int64, c_int64, c_int64, c_int64, c_int64, _p, _p, _p],
    "bl_layernorm_split3": [_p, c_int64, c_int64, _p, _p, c_float, _p, _p],
    "bl_adaln_modulate_split3": [_p, _p, _p, _p, c_int64, c_int64, c_float, _p],
    "bl_diffusion_epilogue_split3": [_p, _p, _p, _p, c_int64, c_int64, c_int, _p],
}
_RESTYPES = {"bl_last_error": ctypes.c_char_p}

_lib = None


def load():
    """Load the shared library (once) and declare every signature."""
    global _lib
    if _lib is None:
        if not LIBRARY_PATH.exists():
            raise RuntimeError(
                f"{LIBRARY_PATH} is missing: build it with `python -m boltz_lumi_b200.build` "
                "(the pair-path kernels have no fallback)"
            )
        lib = ctypes.CDLL(str(LIBRARY_PATH))
        for name, argtypes in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.argtypes = argtypes
            fn.restype = _RESTYPES.get(name, c_int)
        _lib = lib
    return _lib


class CallObserver:
    """Optional hook around every C-ABI call: counts calls and, for the entry
    points in ``timed``, records CUDA events on the launching stream.  Used by
    the benchmark to count launches and time the dominant kernel in place."""

    def __init__(self, timed=()):
        self.timed = set(timed)
        self.calls = 0
        self.records = []  # (name, args, start_event, end_event)

    def before(self, name, args):
        self.calls += 1
        if name in self.timed or "*" in self.timed:
            start = torch.cuda.Event(enable_timing=True)
            start.record()
            return start
        return None

    def after(self, name, args, start):
        if start is not None:
            end = torch.cuda.Event(enable_timing=True)
            end.record()
            self.records.append((name, args, start, end))


_observer = None
_functions = {}  # name -> bound ctypes function


def set_observer(observer):
    """Install (or with None remove) a CallObserver; returns the previous one."""
    global _observer
    previous, _observer = _observer, observer
    return previous


def call(name, *args):
    """Call ``name`` and raise ``RuntimeError`` with the library's message on failure."""
    fn = _functions.get(name)
    if fn is None:
        fn = _functions[name] = getattr(load(), name)
    observer = _observer
    token = observer.before(name, args) if observer is not None else None
    status = fn(*args)
    if observer is not None:
        observer.after(name, args, token)
    if status != 0:
        message = load().bl_last_error().decode(errors="replace")
        raise RuntimeError(f"{name} failed with status {status}: {message}")
    return status


# torch's raw current-stream query: one C call instead of building a
# torch.cuda.Stream object per launch (about 10 us of host time each).
_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def stream_of(tensor: torch.Tensor) -> int:
    """Raw handle of torch's current stream on the tensor's device."""
    if _raw_stream is not None:
        index = tensor.device.index
        return _raw_stream(torch.cuda.current_device() if index is None else index)
    return torch.cuda.current_stream(tensor.device).cuda_stream


def current_stream_handle() -> int:
    """Raw handle of torch's current stream on the current device."""
    if _raw_stream is not None:
        return _raw_stream(torch.cuda.current_device())
    return torch.cuda.current_stream().cuda_stream


def ptr(tensor):
    return None if tensor is None else tensor.data_ptr()


def dtype_code(dtype: torch.dtype) -> int:
    if dtype == torch.float32:
        return BL_F32
    if dtype == torch.bfloat16:
        return BL_BF16
    raise TypeError(f"unsupported dtype {dtype}; expected float32 or bfloat16")


def int64_array(values):
    return (c_int64 * len(values))(*values)


def device_status(reset=False) -> int:
    """Device-side status word (0 = every bounded wait completed)."""
    return load().bl_device_status(1 if reset else 0)
