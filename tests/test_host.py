"""CPU tests of the host layer and the C ABI (no GPU): input contract, criterion, selection,
planning, storage preparation, and that the library exports everything the header declares.

Mirrors the reference's validation/test_ffn.py InputTests / MetricTests / CompositionTests
(test_selection) where the behaviour is shared.
"""
import ctypes
import re
import subprocess
import tempfile
from pathlib import Path

import numpy as np
import pytest
import torch

from ffn_optim_b200 import (DependencyUnavailable, NotApplicable, Selection, compare, ffn, make_plan,
                            problem_from_shapes, validate_tensors)
from ffn_optim_b200 import _lib
from ffn_optim_b200 import cases as C
from ffn_optim_b200.host.inputs import prepare_storage
from oracle import ffn_oracle as O

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "ffn_b200.h"


# ---------------------------------------------------------------- input contract
def test_ranks_and_storage():
    """Ranks 2-8 x fp16/bf16 with stride-2 inputs: storage holds the same rows and the
    oracle on storage equals the oracle on the original tensors (reference test_ffn.py:31-48)."""
    for dtype in (torch.float16, torch.bfloat16):
        for rank in range(2, 9):
            shape = (1,) * (rank - 2) + (3, 17)
            x = torch.randn((*shape[:-1], 34)).to(dtype)[..., ::2]
            w1 = torch.randn(19, 34).to(dtype)[:, ::2]
            w2 = torch.randn(23, 38).to(dtype)[:, ::2]
            p = validate_tensors(x, w1, w2)
            plan = make_plan(p, sm_count=148)
            x2d, a, b, hidden, out, ws, cnt, flg, st = prepare_storage(x, w1, w2, plan)
            for t, rows in ((x2d, p.m), (a, p.h), (b, p.n), (hidden, p.m), (out, p.m)):
                assert t.shape[0] == rows and t.stride(0) % 8 == 0 and t.stride(1) == 1
            dt = p.dtype
            f = lambda t: t.float().numpy()  # noqa: E731
            got = O.ffn(f(x2d[:, :p.k]), f(a[:, :p.k]), f(b[:, :p.h]), dt, staged=True)
            ref = O.ffn(f(x.reshape(p.m, p.k)), f(w1), f(w2), dt, staged=True)
            assert np.array_equal(got, ref)
            assert p.output_shape == (*shape[:-1], 23)
            assert int(cnt.abs().sum()) == 0 and int(flg.abs().sum()) == 0 and int(st.abs().sum()) == 0


def test_invalid_shapes():
    for args in [([3], [4, 3], [3, 4]), ([0, 3], [4, 3], [3, 4]), ([2, 3], [4, 2], [3, 4]),
                 ([1] * 9, [4, 1], [3, 4]), ([True, 3], [4, 3], [3, 4]), ([2, 65536], [4, 65536], [3, 4])]:
        with pytest.raises(ValueError):
            problem_from_shapes(*args)
    for kwargs in ({"dtype": "float32"}, {"layout": "canonical"}):
        with pytest.raises(ValueError):
            problem_from_shapes([2, 3], [4, 3], [3, 4], **kwargs)


def test_no_cpu_fallback():
    with pytest.raises(ValueError, match="requires CUDA"):
        ffn(torch.zeros(2, 3).half(), torch.zeros(4, 3).half(), torch.zeros(3, 4).half())


def test_invalid_tensors():
    x, a, b = torch.zeros(2, 3).half(), torch.zeros(4, 3).half(), torch.zeros(3, 4).half()
    with pytest.raises(ValueError):
        validate_tensors(x, a.float(), b)
    with pytest.raises(ValueError):
        validate_tensors(x.requires_grad_(), a, b)
    with pytest.raises(TypeError):
        validate_tensors(x.detach().numpy(), a, b)


# ---------------------------------------------------------------- criterion
def test_bad_results():
    a = torch.ones(2, 3).half()
    assert compare(a, a)["passed"] and compare(a, a, strict=True)["passed"]
    for bad in (a.float(), a.T, a * float("nan"), a * float("inf"), a * 2):
        assert not compare(bad, a)["passed"]


def test_max_abs_bound_is_strict_only():
    gold = torch.linspace(-1, 1, 1000).half()
    out = gold.clone()
    out[0] += 0.5  # one large error: mean_rel small, max_abs over 2e-2 * max|golden|
    r = compare(out, gold)
    assert r["passed"] and not r["max_abs_ok"] and not compare(out, gold, strict=True)["passed"]


# ---------------------------------------------------------------- selection and planning
def test_selection():
    with pytest.raises(DependencyUnavailable):
        Selection(down_impl="full_load_b").require_available()
    Selection(down_impl="full_load_a").require_available()
    # full_load_a: hidden row block on chip, Y row block in TMEM (256 columns, two halves above
    # that) -> N <= 512 (BASELINE cfg2 and cfg1)
    cfg2 = problem_from_shapes([6993, 100], [1000, 100], [250, 1000])
    plan = make_plan(cfg2, Selection(down_impl="full_load_a"), sm_count=148)
    # 55 row blocks on 148 SMs: clusters of 2 CTAs split each block's 8 H chunks
    assert plan.kernel["variant"] == 9 and plan.block_num == 110 and plan.kernel["tile_n"] == 256
    assert plan.kernel["row_split"] == 2
    assert plan.kernel["up"]["tiles_q"] == 8 and plan.kernel["up"]["k_blocks"] == 2
    small = make_plan(cfg2, Selection(down_impl="full_load_a"), 16, sm_count=148)
    assert small.block_num == 16 and small.kernel["row_split"] == 1
    many = make_plan(problem_from_shapes([512, 256], [1024, 256], [256, 1024]), Selection(down_impl="full_load_a"),
                     sm_count=148)
    assert many.kernel["row_split"] == 8 and many.block_num == 32
    # cfg1: 4 row blocks x 2 Y halves = 8 units, clusters of 8 CTAs split the 16 H chunks
    cfg1 = make_plan(problem_from_shapes([512, 512], [2048, 512], [512, 2048]), Selection(down_impl="full_load_a"),
                     sm_count=148)
    assert cfg1.kernel["variant"] == 9 and cfg1.kernel["row_split"] == 8 and cfg1.block_num == 64
    assert make_plan(problem_from_shapes([512, 512], [2048, 512], [512, 2048]), Selection(down_impl="full_load_a"),
                     63, sm_count=148).kernel["row_split"] == 4
    with pytest.raises(NotApplicable):
        make_plan(problem_from_shapes([512, 512], [2048, 512], [520, 2048]), Selection(down_impl="full_load_a"),
                  sm_count=148)
    with pytest.raises(ValueError):  # a two-phase tile cannot run full_load_a, nor the reverse
        make_plan(cfg2, Selection(down_impl="full_load_a"), sm_count=148, tile="cta128x256")
    with pytest.raises(ValueError):
        make_plan(cfg2, Selection(down_impl="basic"), sm_count=148, tile="rowblock256")
    with pytest.raises(ValueError):
        Selection(up_impl="streamk")
    with pytest.raises(ValueError):
        Selection(down_impl="bogus")
    p = problem_from_shapes([64, 128], [256, 128], [64, 256])
    plan = make_plan(p, Selection(down_impl="streamk"), 8, sm_count=148)
    assert plan.workspace_shape == (2 * 8 * 128, plan.kernel["tile_n"])
    with pytest.raises(NotApplicable):
        make_plan(p, Selection(down_impl="streamk"), 1, sm_count=148)
    with pytest.raises(ValueError):
        make_plan(p, Selection(), 0, sm_count=148)


def _units(phase, C):
    """Python model of the device work list: (cta, tile, kb0, kb1, role)."""
    units = []
    for c in range(C):
        for t in range(c, phase["dp_tiles"], C):
            units.append((c, t, 0, phase["k_blocks"], "full"))
        if phase["sk_tiles"] and c < phase["sk_ctas"]:
            q, r, L = phase["sk_iters"], phase["sk_rem"], phase["k_blocks"]
            st, en = c * q + min(c, r), (c + 1) * q + min(c + 1, r)
            i = st
            while i < en:
                t = i // L
                e = min(en, (t + 1) * L)
                units.append((c, phase["dp_tiles"] + t, i - t * L, e - t * L, "owner" if i == t * L else "contrib"))
                i = e
    return units


def _check_hslice_cover(k, p):
    """Hidden-slice plan: every 128-row hidden block is owned by exactly one CTA (super-block
    sb -> cluster sb mod CL, CTA rank r -> block sb*8 + r), every 128-row n-block of Y by one
    cluster rank, and the partials and counters fit the plan's buffers."""
    S = k["row_split"]
    CL = k["block_num"] // S
    nhb, nnb = k["up"]["tiles_r"], k["down"]["tiles_r"]
    assert S in (2, 4, 8) and k["block_num"] % S == 0 and p.m <= 16 and k["tile_n"] == 16
    sb_n, nbr = -(-nhb // S), -(-nnb // S)
    owned = sorted(sb * S + r for cl in range(CL) for sb in range(cl, sb_n, CL) for r in range(S))
    assert owned == list(range(sb_n * S)) and CL <= sb_n
    assert sorted(r * nbr + j for r in range(S) for j in range(nbr))[:nnb] == list(range(nnb))
    assert k["workspace_floats"] == CL * S * nbr * 128 * 16 and k["counter_words"] == 6 + S
    assert k["up"]["k_blocks"] == -(-p.k // 64) and k["down"]["k_blocks"] == -(-p.h // 64)


@pytest.mark.parametrize("sm", [148, 132])
def test_hslice_plans_fit_the_device(sm):
    """Seeded decode shapes (M <= 16), forced and automatic: every hidden-slice plan covers
    its blocks once, keeps every cluster resident at one CTA per SM (74 / 33 / 15 clusters of
    2 / 4 / 8 on 148 SMs, scaled by the SM count), and its down accumulators fit TMEM beside
    the up accumulator; automatic plans only where the clusters share H evenly."""
    rng = np.random.Generator(np.random.PCG64(sm))
    cap = {2: 74 * sm // 148, 4: 33 * sm // 148, 8: 15 * sm // 148}
    seen = 0
    for _ in range(300):
        m = int(rng.integers(1, 17))
        k = int(rng.integers(1, 65)) * 64
        h = int(rng.integers(1, 400)) * 128 - int(rng.integers(0, 8)) * 8
        n = int(rng.integers(1, 65)) * 64
        p = problem_from_shapes([m, k], [h, k], [n, h])
        for tile in ("hslice16", None):
            try:
                plan = make_plan(p, sm_count=sm, tile=tile)
            except (NotApplicable, ValueError):
                continue
            kk = plan.kernel
            if kk["variant"] != 12:
                assert tile is None
                continue
            seen += 1
            _check_hslice_cover(kk, p)
            S = kk["row_split"]
            CL = kk["block_num"] // S
            nbr = -(-kk["down"]["tiles_r"] // S)
            assert CL <= cap[S] and kk["block_num"] <= sm and nbr * 16 <= 448
            if tile is None:
                sb = -(-kk["up"]["tiles_r"] // S)
                assert sb >= 2 and sb / (-(-sb // CL) * CL) >= 0.85
    assert seen > 100


def test_rowblock_plans_fit_the_device():
    """Seeded shapes with N <= 512 under full_load_a: the Y accumulator is the narrowest of
    64 / 128 / 256 columns that covers N in at most two parts, one unit per (row block,
    part), and the cluster size S of split row blocks follows its doubling rule -- S doubles
    (up to 8) while 2 * S * units CTAs fit the SMs and H has at least 2 * S chunks."""
    rng = np.random.Generator(np.random.PCG64(5))
    for _ in range(300):
        m = int(rng.integers(1, 20000))
        k = int(rng.integers(1, 33)) * 32
        h = int(rng.integers(1, 65)) * 128
        n = int(rng.integers(1, 65)) * 8
        p = problem_from_shapes([m, k], [h, k], [n, h])
        kk = make_plan(p, Selection(down_impl="full_load_a"), sm_count=148).kernel
        ny = kk["tile_n"]
        assert ny == (64 if n <= 64 else (128 if n <= 128 else 256))
        parts = -(-n // ny)
        assert parts <= 2
        units = -(-m // 128) * parts
        chunks = kk["up"]["tiles_q"]
        assert chunks == -(-h // 128) and kk["up"]["tiles_r"] == -(-m // 128)
        S = kk["row_split"]
        assert S in (1, 2, 4, 8) and kk["block_num"] <= 148
        if S > 1:  # the last doubling was allowed
            assert kk["block_num"] == units * S and units * S <= 148 and chunks >= S
        else:
            assert kk["block_num"] == min(units, 148)
        assert S == 8 or 2 * S * units > 148 or chunks < 2 * S  # and the next one was not


@pytest.mark.parametrize("case_id", [c["case_id"] for c in C.load_cases()])
@pytest.mark.parametrize("tile", [None, "pair256x256"])
def test_plan_covers_every_k_block_once(case_id, tile):
    case = C.get_case(case_id)
    p = C.case_problem(case)
    if tile and p.m <= 64:
        pytest.skip("CTA-pair tiles are prefill tiles")
    for down in ("basic", "streamk"):
        try:
            plan = make_plan(p, Selection(down_impl=down), sm_count=148, tile=tile)
        except NotApplicable:
            assert down == "streamk"
            continue
        k = plan.kernel
        if k["variant"] == 12:  # hidden-slice decode: clusters of 8 CTAs over hidden super-blocks
            _check_hslice_cover(k, p)
            continue
        assert k["block_num"] == 148
        owners_n = 148 // (2 if k["cta_pair"] else 1)
        if tile:
            assert k["cta_pair"] == 1 and k["tile_m"] == 256 and k["up"]["tiles_r"] == -(-p.m // 256)
        if p.m <= 16:
            assert k["swap_ab"] == 1 and k["tile_n"] == 16
        elif p.m <= 64:
            assert k["swap_ab"] == 1 and k["tile_n"] == 64
        _check_cover(k, owners_n)
        if down == "basic":
            assert k["down"]["sk_tiles"] == 0


def _check_cover(k, owners_n):
    """Every (tile, k-block) of both phases is computed by exactly one unit and every tile
    has exactly one owner (the CTA that finalises it)."""
    for name in ("up", "down"):
        ph = k[name]
        assert ph["tiles"] == ph["tiles_r"] * ph["tiles_q"]
        cover = {}
        owners = {}
        for c, t, a, b, role in _units(ph, owners_n):
            for kb in range(a, b):
                cover[(t, kb)] = cover.get((t, kb), 0) + 1
            if role in ("full", "owner"):
                owners[t] = owners.get(t, 0) + 1
        assert len(cover) == ph["tiles"] * ph["k_blocks"] and set(cover.values()) == {1}
        assert len(owners) == ph["tiles"] and set(owners.values()) == {1}
        if ph["sk_tiles"]:
            assert 1 <= ph["sk_ctas"] <= owners_n and ph["sk_iters"] >= 8 or ph["sk_ctas"] == 1


def test_prefill_plans_cover_seeded_shapes():
    """The k-block cover and single-owner properties on seeded ragged prefill shapes, for the
    one-CTA and CTA-pair tiles and both down implementations (Stream-K where applicable)."""
    rng = np.random.Generator(np.random.PCG64(9))
    checked = 0
    for _ in range(40):
        m = int(rng.integers(65, 8193))
        k_ = int(rng.integers(1, 257)) * 8
        h = int(rng.integers(1, 1025)) * 8
        n = int(rng.integers(1, 257)) * 8
        p = problem_from_shapes([m, k_], [h, k_], [n, h])
        for tile in (None, "pair256x256"):
            for down in ("basic", "streamk"):
                try:
                    kk = make_plan(p, Selection(down_impl=down), sm_count=148, tile=tile).kernel
                except NotApplicable:
                    assert down == "streamk"
                    continue
                _check_cover(kk, kk["block_num"] // (2 if kk["cta_pair"] else 1))
                checked += 1
    assert checked >= 100


def _claim_model(dp, C, epochs, rng):
    """Python model of the device's dynamic schedule (producer loop of the fused kernel):
    owner c takes tile c first, then claims tile C + (counter - base) until a claim lands at
    or past dp.  Owners run in a random interleaving; returns the tiles per launch and the
    counter."""
    span = max(dp - C, 0) + C
    counter = 0
    launches = []
    for epoch in range(1, epochs + 1):
        base = (epoch - 1) * span
        t_end = max(dp, C) + C
        state = {c: (c, False) for c in range(C)}  # next tile, came from a claim
        done = []
        active = list(range(C))
        while active:
            c = active[rng.integers(len(active))]
            t, claimed = state[c]
            if t >= dp and not claimed:          # no static first tile: one claim
                t, claimed = C + counter - base, True
                counter += 1
            assert not claimed or C <= t < t_end
            if t >= dp:
                active.remove(c)
                continue
            done.append(t)
            state[c] = (C + counter - base, True)
            counter += 1
        launches.append(done)
        assert counter == epoch * span
    return launches, counter


@pytest.mark.parametrize("dp,C", [(0, 4), (3, 8), (8, 8), (9, 8), (1000, 148), (28672, 148), (7, 74)])
def test_dynamic_claims_cover_every_tile_once(dp, C):
    rng = np.random.Generator(np.random.PCG64(dp * 7 + C))
    launches, _ = _claim_model(dp, C, 3, rng)
    for done in launches:
        assert sorted(done) == list(range(dp))


def test_baseline_variants():
    want = {"cfg3_bf16": (1, 16, 12), "cfg4_bf16": (0, 256, 4), "cfg5_bf16": (0, 256, 4), "cfg1_fp16": (0, 128, 1),
            "cfg2_bf16": (0, 128, 1)}
    for cid, (swap, bn, variant) in want.items():
        case = C.get_case(cid)
        plan = make_plan(C.case_problem(case), Selection(down_impl=case["down_impl"]), sm_count=148)
        assert (plan.kernel["swap_ab"], plan.kernel["tile_n"], plan.kernel["variant"]) == (swap, bn, variant), cid
    # cfg5 prefill: CTA pairs, wave-synchronised static order, raster groups of 4 pair rows
    k5 = make_plan(C.case_problem(C.get_case("cfg5_bf16")), Selection(), sm_count=148).kernel
    assert k5["cta_pair"] == 1 and k5["schedule"] == 3 and k5["up"]["group"] == 4 and k5["tile_m"] == 256
    # the reference's block_num=8 keeps one-CTA tiles for small runs, pairs for long ones
    assert make_plan(C.case_problem(C.get_case("cfg1_fp16")), Selection(), 8, sm_count=148).kernel["cta_pair"] == 0
    # cfg3 decode: 32 clusters of 4 CTAs (16 clusters of 8 do not fit one wave: a B200 holds
    # 15), each CTA owning 128 of the 16384 hidden rows
    case = C.get_case("cfg3_bf16")
    k = make_plan(C.case_problem(case), Selection(down_impl="streamk"), sm_count=148).kernel
    assert k["block_num"] == 128 and k["row_split"] == 4
    # 8192 hidden rows: 8 clusters of 8; 40000: no single wave, the most even share (8: 40 / 45)
    p8 = problem_from_shapes([16, 4096], [8192, 4096], [4096, 8192])
    assert make_plan(p8, Selection(), sm_count=148).kernel["row_split"] == 8
    p40 = problem_from_shapes([3, 136], [40000, 136], [200, 40000])
    k40 = make_plan(p40, Selection(), sm_count=148, tile="hslice16").kernel
    assert k40["row_split"] == 8 and k40["block_num"] == 120
    # not for 17 tokens or a single super-block; forced where the swap16 tile applies
    for m, h, gelu, tile, want_v in ((17, 16384, "rational", None, 3), (16, 1024, "rational", None, 2),
                                     (5, 1000, "erf", "hslice16", 12), (1, 64, "rational", "hslice16", 12)):
        p = problem_from_shapes([m, 4096], [h, 4096], [4096, h])
        k = make_plan(p, Selection(down_impl="basic"), sm_count=148, gelu=gelu, tile=tile).kernel
        assert k["variant"] == want_v, (m, h, gelu, tile)
    with pytest.raises(ValueError):
        make_plan(problem_from_shapes([17, 4096], [16384, 4096], [4096, 16384]), Selection(), sm_count=148,
                  tile="hslice16")


# ---------------------------------------------------------------- the C ABI
def _declared():
    text = HEADER.read_text()
    return re.findall(r"FFN_B200_EXPORT\s+[\w\s\*]+?\b(ffn_b200_\w+)\s*\(", text)


def test_library_exports_every_declared_symbol(lib):
    names = _declared()
    assert len(names) >= 13
    assert set(names) == set(_lib.EXPORTED)
    for name in names:
        assert hasattr(lib, name), name
    assert lib.ffn_b200_abi_version() == 2
    assert lib.ffn_b200_strerror(2).decode().startswith("Stream-K")


def test_ctypes_structs_match_the_header():
    src = f'''#include <stdio.h>
#include <stddef.h>
#include "{HEADER}"
int main(void) {{
  printf("%zu %zu %zu %zu\\n", sizeof(ffn_b200_problem), sizeof(ffn_b200_plan), sizeof(ffn_b200_buffers),
         offsetof(ffn_b200_plan, workspace_floats));
  return 0;
}}'''
    with tempfile.TemporaryDirectory() as d:
        c, exe = Path(d) / "s.c", Path(d) / "s"
        c.write_text(src)
        subprocess.run(["gcc", "-o", str(exe), str(c)], check=True)
        sizes = [int(v) for v in subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split()]
    assert sizes == [ctypes.sizeof(_lib.Problem), ctypes.sizeof(_lib.PlanInfo), ctypes.sizeof(_lib.Buffers),
                     _lib.PlanInfo.workspace_floats.offset]


def test_c_planner_rejects_bad_problems(lib):
    info = _lib.PlanInfo()
    for m, k, h, n, dt, down in [(0, 8, 8, 8, 1, 0), (8, 70000, 8, 8, 1, 0), (8, 8, 8, 8, 5, 0), (8, 8, 8, 8, 1, 9)]:
        prob = _lib.Problem(m, k, h, n, dt, down, 0, 0, 148)
        assert lib.ffn_b200_make_plan(ctypes.byref(prob), ctypes.byref(info)) == _lib.ERR_INVALID
    prob = _lib.Problem(64, 64, 64, 64, 1, 2, 0, 0, 148)  # full_load_b
    assert lib.ffn_b200_make_plan(ctypes.byref(prob), ctypes.byref(info)) == _lib.ERR_UNAVAILABLE
    prob = _lib.Problem(64, 64, 64, 600, 1, 1, 0, 0, 148)  # full_load_a with N > 512
    assert lib.ffn_b200_make_plan(ctypes.byref(prob), ctypes.byref(info)) == _lib.ERR_NOT_APPLICABLE
    # prepare without a usable device fails cleanly (no GPU in the CPU suite, or bad pointers)
    bufs = _lib.Buffers()
    h = ctypes.c_void_p()
    prob = _lib.Problem(64, 64, 64, 64, 1, 0, 0, 0, 148)
    assert lib.ffn_b200_prepare(ctypes.byref(prob), ctypes.byref(bufs), 0, ctypes.byref(h)) != 0


def test_swiglu_packing_and_plan(lib):
    """SwiGLU's packed W1: ffn_b200_swiglu_rows, the two row orders of pack_swiglu (checked on
    CPU tensors against an index restatement), and the up GEMM planned over the packed rows."""
    from ffn_optim_b200.host.inputs import pack_swiglu

    assert lib.ffn_b200_swiglu_rows(520, 0) == 128 * 9 and lib.ffn_b200_swiglu_rows(520, 1) == 1040
    assert lib.ffn_b200_swiglu_rows(0, 0) == 0
    h, k = 130, 24
    w1 = torch.arange(2 * h * k, dtype=torch.float32).reshape(2 * h, k).to(torch.bfloat16)
    for swap in (0, 1):
        packed = pack_swiglu(w1, h, swap)
        assert packed.shape == (lib.ffn_b200_swiglu_rows(h, swap), k)
        for r in range(packed.shape[0]):
            if swap:
                src = (r % 2) * h + r // 2
            else:
                i = (r // 128) * 64 + r % 64  # hidden column of the row
                src = (h + i if (r // 64) % 2 else i) if i < h else None
            want = w1[src] if src is not None else torch.zeros(k, dtype=w1.dtype)
            assert torch.equal(packed[r], want), (swap, r)
    info = _lib.PlanInfo()
    for tile, rows, swap in ((1, 128 * 9, 0), (3, 1040, 1)):  # cta128x256, swap16
        prob = _lib.Problem(16, 64, 520, 64, 1, 0, _lib.GELU_CODES["swiglu"], 0, 148, tile)
        assert lib.ffn_b200_make_plan(ctypes.byref(prob), ctypes.byref(info)) == _lib.OK
        assert info.swap_ab == swap
        up = info.up.tiles_r if swap else info.up.tiles_q
        assert up == -(-rows // (128 if swap else info.tile_n))
    prob = _lib.Problem(16, 64, 520, 64, 1, 1, _lib.GELU_CODES["swiglu"], 0, 148)  # full_load_a
    assert lib.ffn_b200_make_plan(ctypes.byref(prob), ctypes.byref(info)) == _lib.OK
    assert info.up.tiles_q == 9 and info.swap_ab == 0  # 64 hidden columns per 128-row chunk


def test_handle_setters_reject_null_and_bad_values(lib):
    assert lib.ffn_b200_set_launch_overlap(None, 1) == _lib.ERR_INVALID
    assert lib.ffn_b200_set_wait_limit(None, 1000) == _lib.ERR_INVALID
    assert lib.ffn_b200_set_trace(None, None) == _lib.ERR_INVALID


def test_canonical_layout_rules_on_host():
    """The shape contract keeps the reference's V1 rule (Linear only); prepare_ffn accepts
    Canonical weights by transposing them, but not with SwiGLU (gate/up are row halves)."""
    from ffn_optim_b200 import prepare_ffn

    with pytest.raises(ValueError):
        problem_from_shapes((4, 8), (8, 16), (16, 4), layout="canonical")
    x, w1, w2 = torch.zeros(4, 8), torch.zeros(8, 32), torch.zeros(16, 4)
    with pytest.raises(ValueError, match="swiglu"):
        prepare_ffn(x, w1, w2, layout="canonical", activation="swiglu")
