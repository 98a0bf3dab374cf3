"""B200-native fused FFN  Y = GELU(X . W1^T) . W2^T  (fp16/bf16, no bias, inference).

Drop-in for the reference's ``ops`` package: ``ffn``, ``prepare_ffn`` and
``PreparedFFN.run`` keep its signatures and semantics; the work runs in one persistent
sm_100a kernel reached through the C ABI of ``include/ffn_b200.h``.
"""
from .api import KernelCompilationError, PreparedFFN, ffn, prepare_ffn
from .host.dispatch import DOWN_IMPLS, DependencyUnavailable, NotApplicable, Selection
from .host.inputs import Problem, problem_from_shapes, quantize_weights_fp8, validate_tensors
from .host.tiling import Plan, Tile, make_plan
from .metrics import compare

__all__ = ["ffn", "prepare_ffn", "PreparedFFN", "quantize_weights_fp8", "KernelCompilationError", "DependencyUnavailable",
           "NotApplicable", "Selection", "DOWN_IMPLS", "Problem", "problem_from_shapes", "validate_tensors",
           "Plan", "Tile", "make_plan", "compare"]
