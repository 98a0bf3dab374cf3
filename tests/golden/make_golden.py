"""Generates the golden fixtures in this directory from the REFERENCE implementation.

    python tests/golden/make_golden.py --reference <path to an hxtsg/ffn_optim checkout>

For every case of ``ffn_optim_b200/configs/cases.json`` it regenerates the seeded inputs
(``ffn_optim_b200.cases``), runs the reference's own torch golden path
``validation/reference.py::ffn_torch`` on CPU, and stores, for a fixed subset of output
rows, the output bit patterns of

  * ``golden``         -- ffn_torch(x, w1, w2)                     (exact-erf GELU, fp32 hidden)
  * ``staged_rational``-- ffn_torch(x, w1, w2, staged=True, rational=True)
                          (the reference kernel's arithmetic: rational GELU, hidden rounded
                          to the input dtype)

together with sha256 digests of the inputs so a test can prove it regenerated the same
inputs.  For the reference's own smoke cases (``configs/v1_cases.json``) it also writes
``ref_<case_id>.npz``: the inputs exactly as the reference's ``common/cases.py::make_inputs``
draws them (its torch.Generator stream; bit patterns of the logical tensors) and the two
outputs above for every row, so the kernel is checked on the reference's own tensors.  ``gelu.npz`` holds the reference's ``gelu_rational`` and torch's exact GELU on
linspace(-10, 10, 10001).  Rows are independent in an FFN, so a row subset pins the
whole computation for those rows.  The fixtures are produced once, here, and committed;
the tests never import the reference.
"""
from __future__ import annotations

import argparse
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
sys.path.insert(0, str(REPO))

from ffn_optim_b200 import cases as C  # noqa: E402

# Output rows kept per case (None = all rows).
ROWS = {
    "cfg1_fp16": "sample:128",
    "cfg2_fp16": "sample:256",
    "cfg2_bf16": "sample:256",
    "cfg4_bf16": "ends:16",
    "cfg5_bf16": "ends:8",
}


def pick_rows(case, m):
    rule = ROWS.get(case["case_id"])
    if rule is None:
        return np.arange(m)
    kind, n = rule.split(":")
    n = int(n)
    if kind == "ends":
        return np.concatenate([np.arange(n), np.arange(m - n, m)])
    rng = np.random.Generator(np.random.PCG64(1234))
    return np.sort(rng.choice(m, size=n, replace=False))


def logical_x_rows(case, rows):
    """Bit patterns [len(rows), K] of the logical X rows (handles the transposed view)."""
    return C.logical_x_rows(case, rows)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of the hxtsg/ffn_optim checkout")
    ap.add_argument("--case", action="append")
    args = ap.parse_args()
    sys.path.insert(0, str(Path(args.reference).resolve()))
    import torch
    from validation.reference import ffn_torch, gelu_rational  # the reference's own code

    torch.manual_seed(0)
    z = torch.linspace(-10, 10, 10001)
    np.savez_compressed(HERE / "gelu.npz", z=z.numpy(), rational=gelu_rational(z).numpy(),
                        exact=torch.nn.functional.gelu(z, approximate="none").numpy())
    print("gelu.npz")

    for case in C.load_cases():
        if args.case and case["case_id"] not in args.case:
            continue
        p = C.case_problem(case)
        dtype = getattr(torch, p.dtype)
        rows = pick_rows(case, p.m)
        xr = logical_x_rows(case, rows)
        w1b, w2b = C.weights(case)
        to_t = lambda b: torch.from_numpy(np.ascontiguousarray(b).view(np.int16)).view(dtype)  # noqa: E731
        x_t, w1_t, w2_t = to_t(xr), to_t(w1b), to_t(w2b)
        with torch.no_grad():
            gold = ffn_torch(x_t, w1_t, w2_t)
            staged = ffn_torch(x_t, w1_t, w2_t, staged=True, rational=True)
        bits = lambda t: t.contiguous().view(torch.int16).numpy().view(np.uint16)  # noqa: E731
        np.savez_compressed(HERE / f"{case['case_id']}.npz", rows=rows.astype(np.int64),
                            x_digest=C.digest(xr), w1_digest=C.digest(w1b), w2_digest=C.digest(w2b),
                            golden=bits(gold), staged_rational=bits(staged), dtype=p.dtype,
                            torch_version=torch.__version__)
        print(case["case_id"], rows.shape, gold.shape)

    # The reference's smoke cases, on the reference's own input stream.
    from common.cases import load_cases as ref_load_cases, make_inputs as ref_make_inputs
    for case in ref_load_cases(Path(args.reference).resolve() / "configs" / "v1_cases.json"):
        if args.case and case["case_id"] not in args.case:
            continue
        x_t, w1_t, w2_t = ref_make_inputs(case)
        with torch.no_grad():
            gold = ffn_torch(x_t, w1_t, w2_t)
            staged = ffn_torch(x_t, w1_t, w2_t, staged=True, rational=True)
        bits = lambda t: t.contiguous().view(torch.int16).numpy().view(np.uint16)  # noqa: E731
        np.savez_compressed(HERE / f"ref_{case['case_id']}.npz", x=bits(x_t), w1=bits(w1_t), w2=bits(w2_t),
                            golden=bits(gold), staged_rational=bits(staged), dtype=case["dtype"],
                            torch_version=torch.__version__)
        print("ref_" + case["case_id"], tuple(x_t.shape), tuple(gold.shape))


if __name__ == "__main__":
    main()
