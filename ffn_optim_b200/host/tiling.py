"""Tiling plan (mirrors ops/host/tiling.py of the reference).

The reference fixes 64x64 output tiles with K steps of 128 and zero-pads M/H/N to 64.
This build plans for the B200 kernel instead: 128-row tcgen05 tiles, 128- or 256-wide
columns (or a swap-AB decode tile of 16/64 tokens), 64-wide K stages, ragged edges masked
by TMA, one persistent CTA per SM.  The planning arithmetic lives in the CUDA library
(``ffn_b200_make_plan``) so the C ABI and this module cannot disagree; it runs on the
host and needs no GPU.
"""
from __future__ import annotations

import ctypes
from dataclasses import asdict, dataclass, field

from .dispatch import DependencyUnavailable, NotApplicable, Selection
from .inputs import Problem, pitch_of

B200_SM_COUNT = 148


def align(value, unit):
    return (value + unit - 1) // unit * unit


@dataclass(frozen=True)
class Tile:
    """One GEMM phase's tile: tm x tn outputs per CTA step, tk = K per pipeline stage."""

    tm: int = 128
    tn: int = 256
    tk: int = 64
    stages: int = 4


@dataclass(frozen=True)
class Plan:
    """Everything one launch needs (reference ops/host/tiling.py:28-55).

    ``block_num`` is the persistent CTA count (<= SM count).  ``up``/``down`` are the two
    phases' tiles; ``kernel`` is the full device schedule from the C planner (tile grids,
    Stream-K split, scratch sizes).  ``workspace_shape`` is the fp32 Stream-K scratch
    ([2 phases * block_num * tile_m, tile_n]).  ``mp/kp/hp/np`` are the row pitches (in
    elements) of X/W1, hidden and Y rows -- the kernel masks ragged tiles, so unlike the
    reference nothing is zero-padded to the tile grid.
    """

    problem: Problem
    selection: Selection
    block_num: int
    up: Tile
    down: Tile
    workspace_shape: tuple
    gelu: str = "rational"
    kernel: dict = field(default_factory=dict)

    @property
    def mp(self):
        return self.problem.m

    @property
    def kp(self):
        return pitch_of(self.problem.k)

    @property
    def hp(self):
        return pitch_of(self.problem.h)

    @property
    def np(self):
        return pitch_of(self.problem.n)

    @property
    def workspace_bytes(self):
        return self.workspace_shape[0] * self.workspace_shape[1] * 4

    def to_dict(self):
        return asdict(self)


def device_sm_count(device=None):
    """SM count of ``device`` (current CUDA device by default); B200's 148 without a GPU."""
    try:
        import torch

        if torch.cuda.is_available():
            return torch.cuda.get_device_properties(device if device is not None else
                                                    torch.cuda.current_device()).multi_processor_count
    except Exception:  # noqa: BLE001 - no usable CUDA runtime: plan for a B200
        pass
    return B200_SM_COUNT


def problem_struct(problem, down_impl, gelu, block_num, sms, tile=None, raster_group=None, l2_policy=None,
                   schedule=None, weight_format=None):
    """The C ABI's ffn_b200_problem for a validated Problem and the tuning overrides."""
    from .. import _lib

    return _lib.Problem(problem.m, problem.k, problem.h, problem.n, _lib.DTYPES[problem.dtype],
                        _lib.DOWN_IMPL_CODES[down_impl], _lib.GELU_CODES[gelu], block_num, sms,
                        _lib.TILE_VARIANTS[tile] if tile else 0, int(raster_group or 0),
                        _lib.L2_POLICIES[l2_policy] if l2_policy else 0,
                        _lib.SCHEDULES[schedule] if schedule else 0,
                        _lib.WEIGHT_FORMATS[weight_format] if weight_format else 0)


def make_plan(problem, selection=Selection(), block_num=None, *, gelu="rational", sm_count=None, tile=None,
              raster_group=None, l2_policy=None, schedule=None, weight_format=None):
    """Plans one fused launch (reference ops/host/tiling.py:58-74).

    ``block_num`` None means one CTA per SM.  ``tile`` None picks the kernel variant
    automatically; a name of ``_lib.TILE_VARIANTS`` forces one (tests, benchmarks).
    ``raster_group`` (tile rows per raster group), ``l2_policy`` ('none' | 'stream_b' | ...)
    and ``schedule`` ('static' | 'dynamic' | 'static_synced' data-parallel tile order) override the
    automatic tuning; ``weight_format='fp8'`` plans the fp8-weight decode tiles (M <= 64,
    otherwise NotApplicable).  Raises
    DependencyUnavailable for the full-load variants, NotApplicable for Stream-K without a
    tail wave (the reference's rule, applied to this kernel's tile grid), ValueError
    otherwise.
    """
    from .. import _lib

    selection.require_available()
    sms = int(sm_count) if sm_count else device_sm_count()
    if block_num is None:
        block_num = sms
    if type(block_num) is not int or not 1 <= block_num <= 65535:
        raise ValueError("block_num must be a positive integer; hardware limit checked before launch")
    if gelu not in _lib.GELU_CODES:
        raise ValueError(f"gelu must be one of {sorted(_lib.GELU_CODES)}")
    if tile is not None and tile not in _lib.TILE_VARIANTS:
        raise ValueError(f"tile must be None or one of {sorted(_lib.TILE_VARIANTS)}")
    if l2_policy is not None and l2_policy not in _lib.L2_POLICIES:
        raise ValueError(f"l2_policy must be None or one of {sorted(_lib.L2_POLICIES)}")
    if raster_group is not None and (type(raster_group) is not int or raster_group < 1):
        raise ValueError("raster_group must be a positive integer")
    if schedule is not None and schedule not in _lib.SCHEDULES:
        raise ValueError(f"schedule must be None or one of {sorted(_lib.SCHEDULES)}")
    if weight_format is not None and weight_format not in _lib.WEIGHT_FORMATS:
        raise ValueError(f"weight_format must be None or one of {sorted(_lib.WEIGHT_FORMATS)}")
    lib = _lib.load()
    prob = problem_struct(problem, selection.down_impl, gelu, block_num, sms, tile, raster_group, l2_policy, schedule,
                          weight_format)
    info = _lib.PlanInfo()
    rc = lib.ffn_b200_make_plan(ctypes.byref(prob), ctypes.byref(info))
    if rc == _lib.ERR_NOT_APPLICABLE:
        if weight_format == "fp8":
            raise NotApplicable("fp8 weights: decode tiles only (M <= 64, even K and H, down_impl basic or streamk)")
        if selection.down_impl == "full_load_a":
            raise NotApplicable("full_load_a keeps a 128 x N fp32 row block in TMEM: needs N <= 512 (two 256-column halves)")
        raise NotApplicable("Stream-K candidate has no remainder tiles for this block_num "
                            "or fewer than two K tiles")
    if rc == _lib.ERR_UNAVAILABLE:
        raise DependencyUnavailable(f"{selection.down_impl}: not implemented in this build")
    if rc != _lib.OK:
        raise ValueError(f"make_plan: {_lib.strerror(rc)}")
    kernel = info.to_dict()
    up = Tile(info.tile_m, info.tile_n, info.tile_k, info.stages)
    down = Tile(info.tile_m, info.tile_n, info.tile_k, info.stages)
    ws_shape = (2 * info.block_num * 128, info.tile_n)
    kernel["overrides"] = {"tile": tile, "raster_group": raster_group, "l2_policy": l2_policy, "schedule": schedule,
                           "weight_format": weight_format}
    return Plan(problem, selection, info.block_num, up, down, ws_shape, gelu, kernel)
