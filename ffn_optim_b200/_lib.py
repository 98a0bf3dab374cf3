"""ctypes binding of the C ABI in ``include/ffn_b200.h`` (library ``_lib/libffn_b200.so``).

This is the whole boundary between the Python host layer and the CUDA code: plain
pointers, sizes and enums, no torch types.  Loading the library needs no GPU; planning
(``make_plan``) runs on the host only.  There is no fallback: if the library is missing
and cannot be built, every entry point raises.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

from . import build as _build

OK = 0
ERR_INVALID = 1
ERR_NOT_APPLICABLE = 2
ERR_UNAVAILABLE = 3
ERR_DEVICE = 4
ERR_CUDA = 5
ERR_ALIGNMENT = 6
ERR_TOO_LARGE = 7
ERR_SCRATCH = 8
NOALLOC_SCRATCH_BYTES = 32 << 20

DTYPES = {"float16": 0, "bfloat16": 1}
DOWN_IMPL_CODES = {"basic": 0, "full_load_a": 1, "full_load_b": 2, "streamk": 3}
GELU_CODES = {"rational": 0, "erf": 1, "silu": 2, "swiglu": 3}  # hidden-layer activation (problem field `gelu`)
# Kernel variants selectable through prepare_ffn(..., tile=...) (None = automatic).
TILE_VARIANTS = {"cta128x256": 1, "cta128x128": 2, "swap16": 3, "swap64": 4, "pair256x256": 5,
                 "swap16k4": 6, "swap64k2": 7, "rowblock64": 8, "rowblock128": 9, "rowblock256": 10,
                 "swap16fp8": 11, "swap64fp8": 12, "hslice16": 13}
WEIGHT_FORMATS = {"native": 0, "fp8": 1}
# Element type of the partial tiles the fused reduce-scatter sends between GPUs.
PARTIAL_TYPES = {"fp32": 0, "input": 1, "fp24": 2}
L2_POLICIES = {"none": 1, "stream_b": 2, "normal": 3, "keep_a": 4}
SCHEDULES = {"static": 1, "dynamic": 2, "static_synced": 3}
KERNEL_ERRORS = {0: "ok", 1: "on-chip pipeline wait timed out", 2: "hidden row-block readiness wait timed out",
                 3: "Stream-K (or cross-cluster) partial wait timed out", 4: "peer GPU partial wait timed out (fused reduce-scatter)",
                 5: "tile claim out of range (counters not reset after an earlier error)",
                 6: "activation beyond the fp16 range of the fp8-weight path (|x| > 65504)"}

# Every symbol the header declares; the CPU tests check the library exports all of them.
EXPORTED = ("ffn_b200_abi_version", "ffn_b200_strerror", "ffn_b200_device_info", "ffn_b200_make_plan",
            "ffn_b200_prepare", "ffn_b200_run", "ffn_b200_rebind_io", "ffn_b200_reset",
            "ffn_b200_set_wait_limit", "ffn_b200_set_fault_injection", "ffn_b200_set_trace",
            "ffn_b200_set_launch_overlap",
            "ffn_b200_set_owner_map", "ffn_b200_get_owner_map", "ffn_b200_quantize_fp8_rows", "ffn_b200_get_plan", "ffn_b200_swiglu_rows",
            "ffn_b200_destroy", "ffn_b200_launch", "ffn_b200_run_noalloc", "ffn_b200_peer_alloc",
            "ffn_b200_peer_open", "ffn_b200_peer_close", "ffn_b200_peer_free", "ffn_b200_reduce_scatter_bytes",
            "ffn_b200_set_reduce_scatter")


class Problem(ctypes.Structure):
    _fields_ = [("m", ctypes.c_int64), ("k", ctypes.c_int64), ("h", ctypes.c_int64), ("n", ctypes.c_int64),
                ("dtype", ctypes.c_int32), ("down_impl", ctypes.c_int32), ("gelu", ctypes.c_int32),
                ("block_num", ctypes.c_int32), ("sm_count", ctypes.c_int32), ("tile_variant", ctypes.c_int32),
                ("raster_group", ctypes.c_int32), ("l2_policy", ctypes.c_int32), ("schedule", ctypes.c_int32),
                ("weight_format", ctypes.c_int32)]


class PhasePlan(ctypes.Structure):
    _fields_ = [(name, ctypes.c_int32) for name in
                ("tiles_r", "tiles_q", "tiles", "k_blocks", "dp_tiles", "sk_tiles", "sk_iters", "sk_rem", "group",
                 "sk_ctas")]

    def to_dict(self):
        return {name: getattr(self, name) for name, _ in self._fields_}


class PlanInfo(ctypes.Structure):
    _fields_ = [("variant", ctypes.c_int32), ("swap_ab", ctypes.c_int32), ("cta_pair", ctypes.c_int32),
                ("tile_m", ctypes.c_int32),
                ("tile_n", ctypes.c_int32), ("tile_k", ctypes.c_int32), ("stages", ctypes.c_int32),
                ("block_num", ctypes.c_int32), ("tmem_cols", ctypes.c_int32), ("smem_bytes", ctypes.c_int64),
                ("up", PhasePlan), ("down", PhasePlan), ("workspace_floats", ctypes.c_int64),
                ("counter_words", ctypes.c_int64), ("flag_words", ctypes.c_int64),
                ("status_words", ctypes.c_int64), ("schedule", ctypes.c_int32), ("row_split", ctypes.c_int32)]

    def to_dict(self):
        out = {}
        for name, _ in self._fields_:
            value = getattr(self, name)
            out[name] = value.to_dict() if isinstance(value, PhasePlan) else value
        return out


class Buffers(ctypes.Structure):
    _fields_ = [("x", ctypes.c_void_p), ("ldx", ctypes.c_int64), ("w1", ctypes.c_void_p), ("ldw1", ctypes.c_int64),
                ("w2", ctypes.c_void_p), ("ldw2", ctypes.c_int64), ("hidden", ctypes.c_void_p),
                ("ldh", ctypes.c_int64), ("y", ctypes.c_void_p), ("ldy", ctypes.c_int64),
                ("workspace", ctypes.c_void_p), ("counters", ctypes.c_void_p), ("flags", ctypes.c_void_p),
                ("status", ctypes.c_void_p),
                ("w1_scale", ctypes.c_void_p), ("w2_scale", ctypes.c_void_p),
                ("bias1", ctypes.c_void_p), ("bias2", ctypes.c_void_p)]


_lock = threading.Lock()
_lib = None


def library_path() -> Path:
    return _build.LIB


def load(build_if_missing: bool = True) -> ctypes.CDLL:
    """Loads (building first when the sources changed and nvcc exists) the CUDA library."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = _build.LIB
        if build_if_missing and not _build.up_to_date():
            try:
                _build.build()
            except RuntimeError:
                if not path.exists():
                    raise
        if not path.exists():
            raise FileNotFoundError(f"ffn_b200 CUDA library not built: {path}")
        lib = ctypes.CDLL(str(path))
        vp, i32, i64, u64 = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_uint64
        sigs = {
            "ffn_b200_abi_version": ([], i32),
            "ffn_b200_strerror": ([i32], ctypes.c_char_p),
            "ffn_b200_device_info": ([i32, ctypes.POINTER(i32), ctypes.POINTER(i32), ctypes.POINTER(i32)], i32),
            "ffn_b200_make_plan": ([ctypes.POINTER(Problem), ctypes.POINTER(PlanInfo)], i32),
            "ffn_b200_prepare": ([ctypes.POINTER(Problem), ctypes.POINTER(Buffers), i32, ctypes.POINTER(vp)], i32),
            "ffn_b200_run": ([vp, vp], i32),
            "ffn_b200_rebind_io": ([vp, vp, vp], i32),
            "ffn_b200_reset": ([vp, vp], i32),
            "ffn_b200_set_wait_limit": ([vp, u64], i32),
            "ffn_b200_set_fault_injection": ([vp, i32], i32),
            "ffn_b200_set_trace": ([vp, vp], i32),
            "ffn_b200_set_launch_overlap": ([vp, i32], i32),
            "ffn_b200_set_owner_map": ([vp, vp], i32),
            "ffn_b200_get_owner_map": ([vp, vp, i32, vp], i32),
            "ffn_b200_quantize_fp8_rows": ([vp, i64, i32, i64, i64, vp, i64, vp, vp], i32),
            "ffn_b200_get_plan": ([vp, ctypes.POINTER(PlanInfo)], i32),
            "ffn_b200_swiglu_rows": ([i64, i32], i64),
            "ffn_b200_destroy": ([vp], i32),
            "ffn_b200_launch": ([ctypes.POINTER(Problem), ctypes.POINTER(Buffers), vp], i32),
            "ffn_b200_run_noalloc": ([ctypes.POINTER(Problem), vp, i64, vp, i64, vp, i64, vp, i64, vp, vp], i32),
            "ffn_b200_peer_alloc": ([u64, ctypes.POINTER(vp), vp], i32),
            "ffn_b200_peer_open": ([vp, ctypes.POINTER(vp)], i32),
            "ffn_b200_peer_close": ([vp], i32),
            "ffn_b200_peer_free": ([vp], i32),
            "ffn_b200_reduce_scatter_bytes": ([vp, i32, i32, ctypes.POINTER(u64), ctypes.POINTER(u64)], i32),
            "ffn_b200_set_reduce_scatter": ([vp, i32, i32, i32, ctypes.POINTER(vp), ctypes.POINTER(vp), vp, i64], i32),
        }
        for name, (args, res) in sigs.items():
            fn = getattr(lib, name)
            fn.argtypes = args
            fn.restype = res
        _lib = lib
        return lib


def strerror(code: int) -> str:
    return load().ffn_b200_strerror(code).decode()
