"""Implementation selection: no silent fallbacks (mirrors ops/host/dispatch.py).

``DOWN_IMPLS`` and the error types keep the reference's names and meaning.  Where the
reference compiles a CATLASS DSL kernel (dispatch.py:97-116), this build binds the
prebuilt sm_100a library through its C ABI instead.
"""
from __future__ import annotations

from dataclasses import dataclass

DOWN_IMPLS = ("basic", "full_load_a", "full_load_b", "streamk")
KERNEL_ENTRIES = {"basic": "ffn_fused_kernel (down: data-parallel tiles)",
                  "streamk": "ffn_fused_kernel (down: data-parallel waves + Stream-K tail)",
                  "full_load_a": "ffn_rowblock_kernel (hidden row block resident on chip, N <= 512)"}


class DependencyUnavailable(RuntimeError):
    """A candidate implementation is not wired in (reference dispatch.py:22-29)."""


class NotApplicable(ValueError):
    """A candidate does not apply to this shape / CTA count (reference dispatch.py:32-39)."""


@dataclass(frozen=True)
class Selection:
    """Up/down implementation names (reference dispatch.py:42-66).

    ``up_impl`` must be 'basic'; ``down_impl`` one of :data:`DOWN_IMPLS`.  'full_load_a'
    (hidden row block resident on chip) applies when N <= 512 and otherwise raises
    :class:`NotApplicable` at planning; 'full_load_b' raises :class:`DependencyUnavailable`
    from :meth:`require_available`.
    """

    up_impl: str = "basic"
    down_impl: str = "basic"

    def __post_init__(self):
        if self.up_impl != "basic":
            raise ValueError("up_impl must be basic")
        if self.down_impl not in DOWN_IMPLS:
            raise ValueError(f"Unknown down_impl: {self.down_impl}")

    def require_available(self):
        if self.down_impl == "full_load_b":
            raise DependencyUnavailable(f"{self.down_impl}: not implemented in this build; no fallback")
        return self


def kernel_provenance(down_impl="basic"):
    """Library path, ABI version and source digest of the kernel that will run."""
    from .. import _lib, build

    Selection(down_impl=down_impl).require_available()
    lib = _lib.load()
    return {"library": str(build.LIB), "abi_version": int(lib.ffn_b200_abi_version()),
            "source_sha256": build.source_digest(), "down_impl": down_impl,
            "entry_point": KERNEL_ENTRIES[down_impl]}
