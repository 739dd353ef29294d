"""ctypes binding of ``include/cpgemm.h`` (the C ABI of ``libcpgemm.so``).

The library must have been built in-tree (``__graft_entry__.build()`` or ``python -m
cutedsl_pingpong_gemm_b200._build``).  There is no fallback: if the library is missing or fails
to load, every entry point raises ``CpgError``.
"""
import ctypes
import os
import threading

from . import _build

CPG_OK = 0
CPG_ERR_INVALID_CONFIG = -1
CPG_ERR_INVALID_SHAPE = -2
CPG_ERR_ALIGNMENT = -3
CPG_ERR_DTYPE = -4
CPG_ERR_UNSUPPORTED = -5
CPG_ERR_NO_DEVICE = -6
CPG_ERR_CUDA = -7
CPG_ERR_DEVICE_TIMEOUT = -8
CPG_ERR_SMEM = -9
CPG_ERR_NULL = -10

CPG_DTYPE_BF16 = 0
CPG_DTYPE_E4M3 = 1
CPG_DTYPE_F32 = 2

CPG_SCALE_TENSOR = 0
CPG_SCALE_BLOCK = 1

CPG_INJECT_SKIP_LOADS = 1
CPG_SPLIT_K_STREAM = -1
CPG_SPLIT_K_HYBRID = -2
CPG_SPLIT_K_DECODE = -3

CPG_ACT_NONE = 0
CPG_ACT_RELU = 1
CPG_ACT_SILU = 2
CPG_ACT_GELU = 3
CPG_ACT_GELU_TANH = 4
ACTIVATIONS = {None: CPG_ACT_NONE, "none": CPG_ACT_NONE, "relu": CPG_ACT_RELU,
               "silu": CPG_ACT_SILU, "gelu": CPG_ACT_GELU, "gelu_tanh": CPG_ACT_GELU_TANH}

ABI_VERSION = 14


class CpgError(RuntimeError):
    """A failed call into libcpgemm; ``code`` is the negative CPG_ERR_* value."""

    def __init__(self, code: int, message: str):
        super().__init__(message)
        self.code = code


class FastDivmodC(ctypes.Structure):
    _fields_ = [("divisor", ctypes.c_int32), ("multiplier", ctypes.c_uint32),
                ("shift_right", ctypes.c_uint32)]


class SchedParamsC(ctypes.Structure):
    _fields_ = [
        ("ncluster_m", ctypes.c_int32), ("ncluster_n", ctypes.c_int32), ("ncluster_l", ctypes.c_int32),
        ("raster_order", ctypes.c_int32),
        ("dm_clusters_per_problem", FastDivmodC),
        ("num_groups_regular", ctypes.c_int32),
        ("dm_group_size", FastDivmodC),
        ("dm_group_size_tail", FastDivmodC),
        ("dm_num_clusters_in_group", FastDivmodC),
        ("cluster_m", ctypes.c_int32), ("cluster_n", ctypes.c_int32),
        ("is_persistent", ctypes.c_int32),
    ]


class GemmConfigC(ctypes.Structure):
    _fields_ = [
        ("tile_m", ctypes.c_int32), ("tile_n", ctypes.c_int32),
        ("epi_tile_m", ctypes.c_int32), ("epi_tile_n", ctypes.c_int32),
        ("cluster_m", ctypes.c_int32), ("cluster_n", ctypes.c_int32), ("cluster_k", ctypes.c_int32),
        ("atom_m", ctypes.c_int32), ("atom_n", ctypes.c_int32),
        ("ab_stage", ctypes.c_int32), ("epi_stage", ctypes.c_int32),
        ("raster_order", ctypes.c_int32),
        ("reuse_ab", ctypes.c_int32), ("is_persistent", ctypes.c_int32),
        ("gemm_n_prologue", ctypes.c_int32),
        ("group_size", ctypes.c_int32),
        ("dynamic_scheduler", ctypes.c_int32),
    ]


class GemmProblemC(ctypes.Structure):
    _fields_ = [
        ("m", ctypes.c_int64), ("n", ctypes.c_int64), ("k", ctypes.c_int64),
        ("lda", ctypes.c_int64), ("ldb", ctypes.c_int64), ("ldd", ctypes.c_int64),
        ("dtype_ab", ctypes.c_int32), ("dtype_d", ctypes.c_int32),
        ("scale_mode", ctypes.c_int32), ("split_k", ctypes.c_int32),
        ("gated", ctypes.c_int32),
        ("l", ctypes.c_int64),
        ("batch_stride_a", ctypes.c_int64), ("batch_stride_b", ctypes.c_int64),
        ("batch_stride_d", ctypes.c_int64),
        ("grouped", ctypes.c_int32),
    ]


class EpilogueC(ctypes.Structure):
    _fields_ = [("alpha", ctypes.c_float), ("bias", ctypes.c_void_p),
                ("scale_a", ctypes.c_void_p), ("scale_b", ctypes.c_void_p),
                ("beta", ctypes.c_float), ("activation", ctypes.c_int32),
                ("source", ctypes.c_void_p), ("ld_source", ctypes.c_int64),
                ("batch_stride_source", ctypes.c_int64)]


CPG_MAX_PEERS = 8


class IpcHandleC(ctypes.Structure):
    _fields_ = [("bytes", ctypes.c_uint8 * 64)]


class ReduceScatterC(ctypes.Structure):
    _fields_ = [("ranks", ctypes.c_int32), ("rank", ctypes.c_int32),
                ("row_start", ctypes.c_int64 * (CPG_MAX_PEERS + 1)), ("ld", ctypes.c_int64),
                ("dst", ctypes.c_void_p * CPG_MAX_PEERS),
                ("count", ctypes.c_void_p * CPG_MAX_PEERS)]


_P = ctypes.POINTER
_i32 = ctypes.c_int32
_i64 = ctypes.c_int64
_vp = ctypes.c_void_p

# name -> (restype, argtypes).  Must list every function declared in include/cpgemm.h.
SIGNATURES = {
    "cpg_config_validate": (ctypes.c_int, [_P(GemmConfigC)]),
    "cpg_gemm_create": (ctypes.c_int, [_P(GemmConfigC), _P(GemmProblemC), ctypes.c_int, _P(_vp)]),
    "cpg_gemm_run": (ctypes.c_int, [_vp, _vp, _vp, _vp, _P(EpilogueC), _vp]),
    "cpg_gemm_run_grouped": (ctypes.c_int, [_vp, _vp, _vp, _vp, _vp, _P(EpilogueC), _vp]),
    "cpg_gemm_destroy": (ctypes.c_int, [_vp]),
    "cpg_gemm_launch_info": (ctypes.c_int, [_vp, _P(_i32), _P(_i32), _P(_i32), _P(_i32), _P(_i32)]),
    "cpg_gemm_sched_params": (ctypes.c_int, [_vp, _P(SchedParamsC)]),
    "cpg_gemm_set_trace": (ctypes.c_int, [_vp, _vp, _i32]),
    "cpg_gemm_set_timeout_ms": (ctypes.c_int, [_vp, _i32]),
    "cpg_gemm_set_fault_injection": (ctypes.c_int, [_vp, _i32]),
    "cpg_gemm_status": (ctypes.c_int, [_vp, _P(_i32)]),
    "cpg_fast_divmod_create": (ctypes.c_int, [_i32, _P(FastDivmodC)]),
    "cpg_fast_divmod_divmod": (ctypes.c_int, [_P(FastDivmodC), _i32, _P(_i32), _P(_i32)]),
    "cpg_fast_divmod_device": (ctypes.c_int, [_P(FastDivmodC), _vp, _vp, _vp, _i64, _vp]),
    "cpg_sched_params_create": (ctypes.c_int, [_i32, _i32, _i32, _i32, _i32, _i32, _i32, _i32, _i32,
                                               _P(SchedParamsC)]),
    "cpg_sched_grid_shape": (ctypes.c_int, [_P(SchedParamsC), _i32, _P(_i32)]),
    "cpg_sched_plan_group_size": (ctypes.c_int, [_P(GemmConfigC), ctypes.c_int64, _i32, _P(_i32)]),
    "cpg_sched_cluster_map": (ctypes.c_int, [_P(SchedParamsC), _P(_i32), _i64]),
    "cpg_sched_cluster_map_device": (ctypes.c_int, [_P(SchedParamsC), _vp, _i64, _vp]),
    "cpg_max_active_clusters": (ctypes.c_int, [_i32, _P(_i32)]),
    "cpg_quantize_e4m3": (ctypes.c_int, [_vp, _i32, _i64, _i64, _i64, _vp, _i64, _vp, _i32, _i32,
                                         _vp]),
    "cpg_cast_f32_bf16": (ctypes.c_int, [_vp, _i64, _i64, _i64, _vp, _i64, _vp, _vp]),
    "cpg_gemm_splitk_static": (ctypes.c_int, [_P(GemmConfigC), _P(GemmProblemC), _vp, _vp, _vp,
                                              _P(EpilogueC), _vp]),
    "cpg_peer_alloc": (ctypes.c_int, [_i64, _P(_vp), _P(IpcHandleC)]),
    "cpg_peer_open": (ctypes.c_int, [_P(IpcHandleC), _P(_vp)]),
    "cpg_peer_close": (ctypes.c_int, [_vp]),
    "cpg_peer_free": (ctypes.c_int, [_vp]),
    "cpg_gemm_run_reduce_scatter": (ctypes.c_int, [_vp, _vp, _vp, _P(ReduceScatterC),
                                                   _P(EpilogueC), _vp]),
    "cpg_gemm_rs_arrivals": (ctypes.c_int, [_vp, _P(ReduceScatterC), _P(ctypes.c_uint32)]),
    "cpg_sched_rs_arrivals": (ctypes.c_int, [_P(SchedParamsC), _i32, _P(ReduceScatterC),
                                             _P(ctypes.c_uint32)]),
    "cpg_peer_finish": (ctypes.c_int, [_vp, _i64, _vp, ctypes.c_uint32, _i64, _i64, _vp, _i64,
                                       _vp, _vp, _i32, _vp]),
    "cpg_strerror": (ctypes.c_char_p, [ctypes.c_int]),
    "cpg_last_error_message": (ctypes.c_char_p, []),
    "cpg_abi_version": (ctypes.c_int, []),
}

_lock = threading.Lock()
_lib = None


def lib_path() -> str:
    return _build.LIB_PATH


def load() -> ctypes.CDLL:
    """Load the in-tree library (never builds implicitly on a GPU box; call build() first)."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = lib_path()
        if not os.path.exists(path):
            raise CpgError(CPG_ERR_NO_DEVICE,
                           f"{path} is missing: build it with __graft_entry__.build() or "
                           f"`python -m cutedsl_pingpong_gemm_b200._build`")
        lib = ctypes.CDLL(path)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        if lib.cpg_abi_version() != ABI_VERSION:
            raise CpgError(CPG_ERR_UNSUPPORTED, f"{path} has ABI {lib.cpg_abi_version()}, "
                                                f"expected {ABI_VERSION}")
        _lib = lib
        return lib


def check(rc: int, what: str = "") -> None:
    if rc == CPG_OK:
        return
    lib = load()
    msg = lib.cpg_last_error_message().decode(errors="replace")
    name = lib.cpg_strerror(rc).decode(errors="replace")
    raise CpgError(rc, f"{what}: {name}: {msg}" if what else f"{name}: {msg}")
