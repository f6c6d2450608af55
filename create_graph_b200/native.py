"""
ctypes binding of libcg_b200.so (declared in include/cg_b200.h).

This is the only module that talks to the sm_100a library. ``lib()`` loads it
once and fails loudly when it is missing or when CUDA is unavailable: the
fused ops have no CPU or library fallback. Every call passes raw device
pointers and the current torch CUDA stream, and raises ``NativeError`` with the
library's message on a non-zero status.
"""

from __future__ import annotations

import ctypes
import functools
import pathlib

import torch

from create_graph_b200.errors import NativeError

LIB_PATH = pathlib.Path(__file__).resolve().parent / "_lib" / "libcg_b200.so"
ABI_VERSION = 1
F32, F64 = 0, 1
ATTN_PRECISIONS = {"fp32": 0, "tf32": 1}  # CG_ATTN_FP32, CG_ATTN_TF32


def attn_precision(name: str) -> int:
    try:
        return ATTN_PRECISIONS[name]
    except KeyError:
        raise ValueError(f"attention precision must be one of {sorted(ATTN_PRECISIONS)}, got {name!r}") from None

_DTYPES = {torch.float32: F32, torch.float64: F64}

i64 = ctypes.c_int64
i32 = ctypes.c_int32
vp = ctypes.c_void_p


class Mat(ctypes.Structure):
    _fields_ = [("ptr", vp), ("sn", i64), ("sh", i64), ("sr", i64)]


class Bias(ctypes.Structure):
    _fields_ = [("ptr", vp), ("sn", i64), ("sh", i64), ("si", i64), ("sj", i64)]


class EdgeAttnArgs(ctypes.Structure):
    _fields_ = [
        ("n", i64),
        ("h", i64),
        ("k", i32),
        ("d", i32),
        ("dtype", i32),
        ("precision", i32),
        ("scale", ctypes.c_double),
        ("key_count", vp),
        ("q", Mat),
        ("k_", Mat),
        ("v", Mat),
        ("bias", Bias),
        ("lse", vp),
        ("grad_out", Mat),
        ("hq", Mat),
        ("hk", Mat),
        ("hv", Mat),
        ("hb", Bias),
        ("out", Mat),
        ("dq", Mat),
        ("dk", Mat),
        ("dv", Mat),
        ("dbias", Bias),
        ("dgrad_out", Mat),
        ("scratch", vp),
        ("token_index", vp),
    ]


class GemmArgs(ctypes.Structure):
    _fields_ = [
        ("m", i64),
        ("n", i64),
        ("k", i64),
        ("a", vp),
        ("lda", i64),
        ("b", vp),
        ("ldb", i64),
        ("c", vp),
        ("ldc", i64),
        ("bias", vp),
        ("aux_in", vp),
        ("aux_out", vp),
        ("ld_aux", i64),
        ("a_mn_major", i32),
        ("b_mn_major", i32),
        ("act", i32),
        ("accumulate", i32),
        ("alpha", ctypes.c_float),
        ("precision", i32),
        ("workspace", vp),
        ("workspace_bytes", i64),
    ]


class PooledAttnArgs(ctypes.Structure):
    _fields_ = [
        ("n", i64),
        ("h", i32),
        ("k", i32),
        ("d", i32),
        ("precision", i32),
        ("scale", ctypes.c_double),
        ("token_index", vp),
        ("key_count", vp),
        ("qkv", vp),
        ("hqkv", vp),
        ("ld_qkv", i64),
        ("bias", vp),
        ("env", vp),
        ("lse", vp),
        ("w", vp),
        ("out", vp),
        ("dout", vp),
        ("hbias", vp),
        ("henv", vp),
        ("dqk", vp),
        ("ld_dqk", i64),
        ("wv", vp),
        ("dbias", vp),
        ("denv", vp),
        ("ddout", vp),
        ("ld_bias", i64),
        ("ld_hbias", i64),
    ]


class GeomArgs(ctypes.Structure):
    _fields_ = [
        ("pos", vp),
        ("nbr", vp),
        ("rev_ptr", vp),
        ("rev_idx", vp),
        ("n_atoms", i64),
        ("k", i32),
        ("n_rbf", i32),
        ("cutoff", ctypes.c_float),
        ("gamma", ctypes.c_float),
    ]


ACT_NONE, ACT_SILU, ACT_SILU_GRAD, ACT_ADD = 0, 1, 2, 3
GEMM_TF32, GEMM_FP32 = 0, 1
f32 = ctypes.c_float
_I = ctypes.c_int

# name -> (restype, argtypes)
_SIGNATURES = {
    "cg_last_error": (ctypes.c_char_p, []),
    "cg_version": (ctypes.c_int, []),
    "cg_launch_count": (i64, []),
    "cg_edge_attn_fwd1": (ctypes.c_int, [ctypes.POINTER(EdgeAttnArgs), vp]),
    "cg_edge_attn_bwd1": (ctypes.c_int, [ctypes.POINTER(EdgeAttnArgs), vp]),
    "cg_edge_attn_bwd2": (ctypes.c_int, [ctypes.POINTER(EdgeAttnArgs), vp]),
    "cg_edge_attn_scratch_bytes": (i64, [ctypes.POINTER(EdgeAttnArgs)]),
    "cg_gemm_tf32": (ctypes.c_int, [ctypes.POINTER(GemmArgs), vp]),
    "cg_gemm_workspace_bytes": (i64, [ctypes.POINTER(GemmArgs)]),
    "cg_gemm_tf32_noalloc": (ctypes.c_int, [ctypes.POINTER(GemmArgs), vp]),
    "cg_device_error": (ctypes.c_int, [ctypes.POINTER(ctypes.c_int), ctypes.c_int]),
    "cg_gather_rows": (_I, [vp, i64, vp, i64, i64, vp, i64, vp]),
    "cg_segment_sum": (_I, [vp, i64, vp, vp, i64, i64, vp, i64, _I, vp]),
    "cg_segment_sum_scaled": (_I, [vp, vp, i64, i64, i32, i32, vp, vp, i64, vp, i64, _I, vp]),
    "cg_pooled_attn_fwd": (_I, [ctypes.POINTER(PooledAttnArgs), vp]),
    "cg_pooled_attn_bwd1": (_I, [ctypes.POINTER(PooledAttnArgs), vp]),
    "cg_pooled_attn_bwd2": (_I, [ctypes.POINTER(PooledAttnArgs), vp]),
    "cg_pooled_attn_out": (_I, [ctypes.POINTER(PooledAttnArgs), vp]),
    "cg_colsum_scratch_bytes": (i64, [i64, i64]),
    "cg_colsum": (_I, [vp, i64, i64, i64, vp, _I, vp, vp]),
    "cg_coldot_scratch_bytes": (i64, [i64, i64]),
    "cg_coldot": (_I, [vp, vp, i64, i64, vp, _I, vp, vp]),
    "cg_silu": (_I, [vp, vp, i64, vp]),
    "cg_silu_grad": (_I, [vp, vp, vp, i64, vp]),
    "cg_silu_grad2": (_I, [vp, vp, vp, vp, i64, vp]),
    "cg_scale_shift": (_I, [vp, vp, vp, vp, i64, i64, vp]),
    "cg_rownorm_fwd": (_I, [vp, i64, i64, f32, vp, vp, vp]),
    "cg_rownorm_bwd1": (_I, [vp, vp, i64, i64, f32, vp, vp]),
    "cg_rownorm_bwd1_add": (_I, [vp, vp, vp, i64, i64, f32, vp, vp]),
    "cg_adamw_step": (_I, [vp, vp, vp, vp, i64, f32, f32, f32, f32, f32, i64, vp]),
    "cg_adamw_step_counted": (_I, [vp, vp, vp, vp, i64, f32, f32, f32, f32, f32, vp, vp]),
    "cg_csr_from_index": (_I, [vp, i64, i64, vp, vp, vp]),
    "cg_rownorm_bwd2": (_I, [vp, vp, vp, i64, i64, f32, vp, vp, vp]),
    "cg_mse_energy_force": (_I, [vp, vp, i64, vp, vp, i64, vp, vp]),
    "cg_mse_energy_force_bwd": (_I, [vp, vp, i64, vp, vp, i64, vp, vp, vp, vp]),
    "cg_pool": (_I, [vp, vp, i64, i64, i64, vp, vp]),
    "cg_pool_outer": (_I, [vp, vp, i64, i64, i64, vp, vp]),
    "cg_pool_dot": (_I, [vp, vp, i64, i64, i64, vp, vp]),
    "cg_edge_geom_fwd": (_I, [ctypes.POINTER(GeomArgs), vp, vp, vp]),
    "cg_edge_geom_bwd1": (_I, [ctypes.POINTER(GeomArgs), vp, vp, vp, vp, vp]),
    "cg_edge_geom_bwd2": (_I, [ctypes.POINTER(GeomArgs), vp, vp, vp, vp, vp, vp, vp, vp]),
    "cg_neighbor_list_workspace": (_I, [i64]),
    "cg_neighbor_list": (_I, [vp, vp, i64, i64, i64, f32, i32, vp, vp, vp, vp, vp, vp]),
}


def exported_symbols() -> list[str]:
    """Every symbol the Python side binds (each one is declared in include/cg_b200.h)."""
    return sorted(_SIGNATURES)


@functools.cache
def load_library() -> ctypes.CDLL:
    """Load libcg_b200.so without touching the GPU (CPU-side checks use this)."""
    if not LIB_PATH.exists():
        raise NativeError(
            f"{LIB_PATH} is missing: build it with `python -m create_graph_b200.build` "
            "(the fused ops have no fallback)"
        )
    lib = ctypes.CDLL(str(LIB_PATH))
    for name, (res, args) in _SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if lib.cg_version() != ABI_VERSION:
        raise NativeError(f"libcg_b200.so has ABI {lib.cg_version()}, expected {ABI_VERSION}")
    return lib


def lib() -> ctypes.CDLL:
    """The library, for a compute call: CUDA must be available."""
    if not torch.cuda.is_available():
        raise NativeError("create_graph_b200 fused ops need a CUDA device (sm_100a); none is visible")
    return load_library()


def check(status: int) -> None:
    if status != 0:
        message = load_library().cg_last_error().decode(errors="replace")
        raise NativeError(message or f"libcg_b200 call failed with status {status}")


def stream_ptr(device: torch.device | None = None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def dtype_code(t: torch.Tensor) -> int:
    try:
        return _DTYPES[t.dtype]
    except KeyError:
        raise NativeError(f"unsupported dtype {t.dtype}: float32 or float64 expected") from None


def require_cuda(*tensors: torch.Tensor) -> None:
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise NativeError(
                "create_graph_b200 fused ops run on CUDA tensors only (no CPU fallback); got a "
                f"{t.device} tensor"
            )


def device_error(reset: bool = False) -> int:
    """The device error word (non-zero: a kernel's bounded wait gave up)."""
    out = ctypes.c_int(0)
    check(lib().cg_device_error(ctypes.byref(out), int(reset)))
    return out.value


def ptr(t: torch.Tensor | None) -> int | None:
    """Device address of a tensor (None for None)."""
    return None if t is None else t.data_ptr()


# entry point name -> list of (start, end, info) CUDA event pairs, for the
# entry points a benchmark asked to time (``time_entry_points``)
TIMED: dict[str, list] = {}


def time_entry_points(names, enable: bool = True) -> None:
    """Record CUDA events around every call of the named entry points."""
    for name in names:
        if enable:
            TIMED.setdefault(name, [])
        else:
            TIMED.pop(name, None)


def invoke(name: str, *args, info=None) -> None:
    """Call a status-returning entry point (the last argument is the stream)."""
    fn = getattr(lib(), name)
    slot = TIMED.get(name)
    if slot is None:
        check(fn(*args))
        return
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    check(fn(*args))
    end.record()
    slot.append((start, end, info))


call = invoke


def launch_count() -> int:
    """Kernels libcg_b200.so has launched in this process."""
    return int(load_library().cg_launch_count())
