"""ctypes binding of ``libavey_b200.so`` (C ABI: ``include/avey_b200.h``).

Loading fails loudly: there is no fallback when the library is missing.
"""

from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / 'lib' / 'libavey_b200.so'

AVEY_F32, AVEY_F16, AVEY_BF16, AVEY_F64 = 0, 1, 2, 3
KERNEL_AUTO, KERNEL_SIMT, KERNEL_TCGEN05 = 0, 1, 2
# AveyPlan.reason: why the tcgen05 kernels were not chosen (0: they were).
REASON_DTYPE, REASON_CONTEXT, REASON_ALIGNMENT, REASON_FORCED, REASON_FEATURES, REASON_SMALL = range(1, 7)
ACTIVATION_IDS = {'identity': 0, 'relu': 1, 'relu2': 2, 'silu': 3, 'gelu': 4}

STATUS_NAMES = {
    0: 'AVEY_OK', -1: 'AVEY_ERR_ARGUMENT', -2: 'AVEY_ERR_ARCH', -3: 'AVEY_ERR_UNSUPPORTED',
    -4: 'AVEY_ERR_LAUNCH', -5: 'AVEY_ERR_DEVICE', -6: 'AVEY_ERR_CUDA',
}

# Exported symbols, mirrored from include/avey_b200.h (tests check the header).
EXPORTS = ('avey_fwd_v1', 'avey_fwd_plan', 'avey_fwd_workspace_size', 'avey_fwd_noalloc_v1',
           'avey_bwd_step_v1', 'avey_bwd_workspace_size',
           'avey_last_error', 'avey_device_status', 'avey_launch_count', 'avey_abi_version',
           'avey_test_hooks_v1', 'avey_gemm_v1', 'avey_fwd_presummed_v1')
BWD_PREP, BWD_SCORES, BWD_EPILOGUE, BWD_DSCORES, BWD_FINAL = range(5)
NOALLOC_MAX_ROWS = 1 << 20
ABI_VERSION = 5


class AveyFwdParams(ctypes.Structure):
    _fields_ = [
        ('struct_size', ctypes.c_uint32),
        ('dtype', ctypes.c_int32),
        ('batch', ctypes.c_int64),
        ('context', ctypes.c_int64),
        ('features', ctypes.c_int64),
        ('z_tr', ctypes.c_void_p),
        ('z_tr_batch_stride', ctypes.c_int64),
        ('z_tr_row_stride', ctypes.c_int64),
        ('v', ctypes.c_void_p),
        ('v_row_stride', ctypes.c_int64),
        ('z_tl', ctypes.c_void_p),
        ('z_tl_batch_stride', ctypes.c_int64),
        ('z_tl_row_stride', ctypes.c_int64),
        ('bias', ctypes.c_void_p),
        ('valid', ctypes.c_void_p),
        ('valid_batch_stride', ctypes.c_int64),
        ('valid_row_stride', ctypes.c_int64),
        ('out', ctypes.c_void_p),
        ('out_batch_stride', ctypes.c_int64),
        ('out_row_stride', ctypes.c_int64),
        ('eps', ctypes.c_double),
        ('norm_eps', ctypes.c_double),
        ('causal', ctypes.c_int32),
        ('normalize', ctypes.c_int32),
        ('activation', ctypes.c_int32),
        ('kernel', ctypes.c_int32),
        ('workspace', ctypes.c_void_p),
        ('workspace_bytes', ctypes.c_uint64),
        ('lengths', ctypes.c_void_p),
    ]


class AveyBwdParams(ctypes.Structure):
    _fields_ = [
        ('struct_size', ctypes.c_uint32),
        ('dtype', ctypes.c_int32),
        ('gemm_dtype', ctypes.c_int32),
        ('causal', ctypes.c_int32),
        ('normalize', ctypes.c_int32),
        ('activation', ctypes.c_int32),
        ('batch', ctypes.c_int64),
        ('context', ctypes.c_int64),
        ('features', ctypes.c_int64),
        ('eps', ctypes.c_double),
        ('norm_eps', ctypes.c_double),
        ('z_tr', ctypes.c_void_p),
        ('z_tr_batch_stride', ctypes.c_int64),
        ('z_tr_row_stride', ctypes.c_int64),
        ('v', ctypes.c_void_p),
        ('v_row_stride', ctypes.c_int64),
        ('z_tl', ctypes.c_void_p),
        ('z_tl_batch_stride', ctypes.c_int64),
        ('z_tl_row_stride', ctypes.c_int64),
        ('bias', ctypes.c_void_p),
        ('valid', ctypes.c_void_p),
        ('valid_batch_stride', ctypes.c_int64),
        ('valid_row_stride', ctypes.c_int64),
        ('grad_out', ctypes.c_void_p),
        ('grad_out_batch_stride', ctypes.c_int64),
        ('grad_out_row_stride', ctypes.c_int64),
        ('zm', ctypes.c_void_p),
        ('norms', ctypes.c_void_p),
        ('g', ctypes.c_void_p),
        ('s', ctypes.c_void_p),
        ('den', ctypes.c_void_p),
        ('num', ctypes.c_void_p),
        ('dnum', ctypes.c_void_p),
        ('dden', ctypes.c_void_p),
        ('ds0', ctypes.c_void_p),
        ('dgsym', ctypes.c_void_p),
        ('dzd', ctypes.c_void_p),
        ('dzh', ctypes.c_void_p),
        ('workspace', ctypes.c_void_p),
        ('workspace_bytes', ctypes.c_uint64),
        ('grad_z_tr', ctypes.c_void_p),
        ('grad_v', ctypes.c_void_p),
        ('grad_z_tl', ctypes.c_void_p),
        ('grad_bias', ctypes.c_void_p),
        ('grad_batch_stride', ctypes.c_int64),
        ('grad_row_stride', ctypes.c_int64),
    ]


class AveyGemmParams(ctypes.Structure):
    _fields_ = [
        ('struct_size', ctypes.c_uint32),
        ('dtype', ctypes.c_int32),
        ('out_dtype', ctypes.c_int32),
        ('mode', ctypes.c_int32),
        ('batch', ctypes.c_int64),
        ('m', ctypes.c_int64),
        ('n', ctypes.c_int64),
        ('k', ctypes.c_int64),
        ('a', ctypes.c_void_p),
        ('a_batch_stride', ctypes.c_int64),
        ('a_ld', ctypes.c_int64),
        ('a_major', ctypes.c_int32),
        ('b', ctypes.c_void_p),
        ('b_batch_stride', ctypes.c_int64),
        ('b_ld', ctypes.c_int64),
        ('b_major', ctypes.c_int32),
        ('c', ctypes.c_void_p),
        ('c_batch_stride', ctypes.c_int64),
        ('c_ld', ctypes.c_int64),
        ('bias', ctypes.c_void_p),
        ('gate', ctypes.c_void_p),
        ('gate_batch_stride', ctypes.c_int64),
        ('gate_ld', ctypes.c_int64),
        ('activation', ctypes.c_int32),
        ('sumsq_col0', ctypes.c_int32),
        ('sumsq', ctypes.c_void_p),
        ('kernel', ctypes.c_int32),
    ]


class AveyPlan(ctypes.Structure):
    _fields_ = [
        ('kernel', ctypes.c_int32),
        ('launches', ctypes.c_int32),
        ('grid', ctypes.c_int32),
        ('block', ctypes.c_int32),
        ('smem_bytes', ctypes.c_int32),
        ('reason', ctypes.c_int32),
    ]


class NativeError(RuntimeError):
    """A non-OK AveyStatus from the library."""

    def __init__(self, status: int, message: str):
        self.status = status
        super().__init__(f'{STATUS_NAMES.get(status, status)}: {message}')


_lock = threading.Lock()
_lib = None


def library_path() -> Path:
    override = os.environ.get('AVEY_B200_LIB')
    return Path(override) if override else LIB_PATH


def lib() -> ctypes.CDLL:
    """The loaded library; raises if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = library_path()
        if not path.exists():
            raise RuntimeError(
                f'avey_kernel_b200: CUDA library not found at {path}. Build it with '
                '`python -m avey_kernel_b200.csrc.build` (there is no CPU fallback).')
        dll = ctypes.CDLL(str(path))
        dll.avey_fwd_v1.argtypes = [ctypes.POINTER(AveyFwdParams), ctypes.c_void_p]
        dll.avey_fwd_v1.restype = ctypes.c_int
        dll.avey_fwd_plan.argtypes = [ctypes.POINTER(AveyFwdParams), ctypes.POINTER(AveyPlan)]
        dll.avey_fwd_plan.restype = ctypes.c_int
        dll.avey_fwd_workspace_size.argtypes = [ctypes.POINTER(AveyFwdParams),
                                                ctypes.POINTER(ctypes.c_uint64)]
        dll.avey_fwd_workspace_size.restype = ctypes.c_int
        dll.avey_fwd_noalloc_v1.argtypes = [ctypes.POINTER(AveyFwdParams), ctypes.c_void_p]
        dll.avey_fwd_noalloc_v1.restype = ctypes.c_int
        dll.avey_bwd_step_v1.argtypes = [ctypes.POINTER(AveyBwdParams), ctypes.c_int,
                                         ctypes.c_void_p]
        dll.avey_bwd_step_v1.restype = ctypes.c_int
        dll.avey_bwd_workspace_size.argtypes = [ctypes.POINTER(AveyBwdParams),
                                                ctypes.POINTER(ctypes.c_uint64)]
        dll.avey_bwd_workspace_size.restype = ctypes.c_int
        dll.avey_last_error.argtypes = []
        dll.avey_last_error.restype = ctypes.c_char_p
        dll.avey_device_status.argtypes = [ctypes.POINTER(ctypes.c_uint32), ctypes.c_int]
        dll.avey_device_status.restype = ctypes.c_int
        dll.avey_launch_count.argtypes = []
        dll.avey_launch_count.restype = ctypes.c_uint64
        dll.avey_abi_version.argtypes = []
        dll.avey_abi_version.restype = ctypes.c_int
        dll.avey_test_hooks_v1.argtypes = [ctypes.c_longlong, ctypes.c_int]
        dll.avey_test_hooks_v1.restype = ctypes.c_int
        dll.avey_gemm_v1.argtypes = [ctypes.POINTER(AveyGemmParams), ctypes.c_void_p]
        dll.avey_gemm_v1.restype = ctypes.c_int
        dll.avey_fwd_presummed_v1.argtypes = [ctypes.POINTER(AveyFwdParams), ctypes.c_void_p,
                                              ctypes.c_int, ctypes.c_void_p]
        dll.avey_fwd_presummed_v1.restype = ctypes.c_int
        if dll.avey_abi_version() != ABI_VERSION:
            raise RuntimeError(f'{path}: ABI version {dll.avey_abi_version()} != {ABI_VERSION}')
        _lib = dll
        return _lib


def _check(status: int) -> None:
    if status != 0:
        msg = lib().avey_last_error().decode(errors='replace')
        raise NativeError(status, msg)


def forward(params: AveyFwdParams, stream: int) -> None:
    _check(lib().avey_fwd_v1(ctypes.byref(params), ctypes.c_void_p(stream)))


def forward_noalloc(params: AveyFwdParams, stream: int) -> None:
    """avey_fwd_noalloc_v1: like forward() but with the library's own scratch."""
    _check(lib().avey_fwd_noalloc_v1(ctypes.byref(params), ctypes.c_void_p(stream)))


def gemm(params: AveyGemmParams, stream: int) -> None:
    """avey_gemm_v1: enqueue one batched tcgen05 matrix product on `stream`."""
    _check(lib().avey_gemm_v1(ctypes.byref(params), ctypes.c_void_p(stream)))


def forward_presummed(params: AveyFwdParams, sumsq: int, planes: int, stream: int) -> None:
    """avey_fwd_presummed_v1: forward with the row sums of squares supplied."""
    _check(lib().avey_fwd_presummed_v1(ctypes.byref(params), ctypes.c_void_p(sumsq), int(planes),
                                       ctypes.c_void_p(stream)))


def plan(params: AveyFwdParams) -> AveyPlan:
    out = AveyPlan()
    _check(lib().avey_fwd_plan(ctypes.byref(params), ctypes.byref(out)))
    return out


def workspace_size(params: AveyFwdParams) -> int:
    out = ctypes.c_uint64(0)
    _check(lib().avey_fwd_workspace_size(ctypes.byref(params), ctypes.byref(out)))
    return int(out.value)


def bwd_step(params: AveyBwdParams, step: int, stream: int) -> None:
    """avey_bwd_step_v1: enqueue one backward step on `stream`."""
    _check(lib().avey_bwd_step_v1(ctypes.byref(params), int(step), ctypes.c_void_p(stream)))


def bwd_workspace_size(params: AveyBwdParams) -> int:
    out = ctypes.c_uint64(0)
    _check(lib().avey_bwd_workspace_size(ctypes.byref(params), ctypes.byref(out)))
    return int(out.value)


def device_status(clear: bool = False) -> int:
    flags = ctypes.c_uint32(0)
    _check(lib().avey_device_status(ctypes.byref(flags), int(clear)))
    return flags.value


def test_hooks(wait_limit_cycles: int = 0, stall: bool = False) -> None:
    """avey_test_hooks_v1 (tests only): lower the bounded-wait limit and make
    the fused kernel's TMA and MMA warps idle so a wait runs out. Call with no
    arguments to restore the defaults."""
    _check(lib().avey_test_hooks_v1(int(wait_limit_cycles), 1 if stall else 0))


def launch_count() -> int:
    return int(lib().avey_launch_count())


def new_bwd_params() -> AveyBwdParams:
    p = AveyBwdParams()
    p.struct_size = ctypes.sizeof(AveyBwdParams)
    return p


def new_params() -> AveyFwdParams:
    p = AveyFwdParams()
    p.struct_size = ctypes.sizeof(AveyFwdParams)
    return p
