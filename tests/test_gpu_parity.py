"""GPU parity of the fused kernel against the reference's golden outputs and the CPU oracle.

* small / medium cases: against tests/golden fixtures (outputs of the reference's own
  ffn_torch) -- the kernel arithmetic (rational GELU, hidden rounded to the input dtype)
  against ``staged_rational`` within two output ulps plus 1e-3 * max|golden|, and against
  the default exact-erf golden with the reference criterion plus the max-abs bound;
* full BASELINE sizes: fixture rows plus random rows checked with the oracle (rows are
  independent), and run-to-run bit identity;
* ragged shapes, swap-AB decode tiles, block_num variants, the drop-in API semantics.
"""
import numpy as np
import pytest
import torch

from ffn_optim_b200 import NotApplicable, compare, prepare_ffn
from ffn_optim_b200 import cases as C
from oracle import ffn_oracle as O

pytestmark = pytest.mark.gpu

GOLDEN = C.CASES_FILE.parents[2] / "tests" / "golden"
SMALL = ["aligned_fp16", "tails_bf16", "rank8_fp16", "cfg1_fp16", "cfg2_fp16", "cfg2_bf16"]


def bits_of(t):
    return t.contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def assert_close_bits(out_bits, gold_bits, dt, floor=1e-3):
    """Kernel vs a golden of the same arithmetic: <= 2 output ulps + floor * max|golden|."""
    o, g = O.from_bits(out_bits, dt), O.from_bits(gold_bits, dt)
    rel = 2.0 ** -6 if dt == "bfloat16" else 2.0 ** -9
    bound = rel * np.abs(g) + floor * np.abs(g).max()
    excess = np.abs(o - g) - bound
    assert np.all(excess <= 0), f"max excess {excess.max()} at {np.unravel_index(excess.argmax(), excess.shape)}"


def assert_criterion(out_bits, gold_bits, dt):
    o = torch.from_numpy(O.from_bits(out_bits, dt))
    g = torch.from_numpy(O.from_bits(gold_bits, dt))
    r = compare(o, g, strict=True)
    assert r["passed"], r


def rows_of(y, rows):
    return bits_of(y.reshape(-1, y.shape[-1])[torch.as_tensor(rows, device=y.device)])


def run(x, w1, w2, **kw):
    prepared = prepare_ffn(x, w1, w2, **kw)
    prepared.set_wait_limit(2.0)
    y = prepared.run()
    prepared.check()
    return prepared, y


@pytest.mark.parametrize("case_id", SMALL)
@pytest.mark.parametrize("down_impl", ["basic", "streamk", "full_load_a"])
def test_small_cases_vs_reference_golden(case_id, down_impl):
    case = C.get_case(case_id)
    fx = np.load(GOLDEN / f"{case_id}.npz")
    dt = str(fx["dtype"])
    x, w1, w2 = C.make_inputs(case, device="cuda")
    try:
        prepared, y = run(x, w1, w2, down_impl=down_impl)
    except NotApplicable:
        assert down_impl == "streamk" or (down_impl == "full_load_a" and case["weight2_shape"][0] > 512)
        pytest.skip(f"{down_impl} not applicable")
    assert tuple(y.shape) == C.case_problem(case).output_shape and y.dtype == x.dtype
    got = rows_of(y, fx["rows"])
    assert_close_bits(got, fx["staged_rational"], dt)
    assert_criterion(got, fx["golden"], dt)


@pytest.mark.parametrize("case_id", ["aligned_fp16", "tails_bf16", "rank8_fp16"])
@pytest.mark.parametrize("down_impl", ["basic", "streamk", "full_load_a"])
def test_reference_smoke_cases_on_reference_inputs(case_id, down_impl):
    """The reference's smoke cases on the tensors the reference itself draws
    (common/cases.py:34-50, restated by ``cases.reference_stream_inputs`` and checked bit for
    bit against the reference-generated fixture ``ref_<case>.npz``), views and all, against
    the reference's ``ffn_torch`` outputs on the same tensors."""
    fx = np.load(GOLDEN / f"ref_{case_id}.npz")
    dt = str(fx["dtype"])
    x, w1, w2 = C.reference_stream_inputs(C.get_case(case_id), device="cuda")
    assert np.array_equal(bits_of(x.contiguous()).reshape(fx["x"].shape), fx["x"])
    try:
        prepared, y = run(x, w1, w2, down_impl=down_impl)
    except NotApplicable:
        assert down_impl == "streamk"
        pytest.skip("Stream-K not applicable")
    assert tuple(y.shape) == fx["golden"].shape and y.dtype == x.dtype
    got = bits_of(y).reshape(-1, fx["golden"].shape[-1])
    assert_close_bits(got, fx["staged_rational"].reshape(got.shape), dt)
    assert_criterion(got, fx["golden"].reshape(got.shape), dt)


@pytest.mark.parametrize("case_id", ["cfg1_fp16", "cfg2_bf16", "tails_bf16"])
def test_erf_gelu_vs_reference_golden(case_id):
    case = C.get_case(case_id)
    fx = np.load(GOLDEN / f"{case_id}.npz")
    dt = str(fx["dtype"])
    x, w1, w2 = C.make_inputs(case, device="cuda")
    _, y = run(x, w1, w2, gelu="erf", down_impl="basic")
    got = rows_of(y, fx["rows"])
    assert_criterion(got, fx["golden"], dt)
    # The unstaged golden keeps the hidden tensor in fp32; the kernel rounds it once.
    assert_close_bits(got, fx["golden"], dt, floor=4e-3)


@pytest.mark.parametrize("down_impl", ["streamk", "basic"])
def test_cfg3_decode_vs_reference_golden(down_impl):
    case = C.get_case("cfg3_bf16")
    fx = np.load(GOLDEN / "cfg3_bf16.npz")
    x, w1, w2 = C.make_inputs(case, device="cuda")
    prepared, y = run(x, w1, w2, down_impl=down_impl)
    assert prepared.plan.kernel["swap_ab"] == 1
    got = bits_of(y)
    assert_close_bits(got, fx["staged_rational"], "bfloat16")
    assert_criterion(got, fx["golden"], "bfloat16")
    y2 = prepared.run()
    prepared.check()
    assert np.array_equal(bits_of(y2), got), "run-to-run results differ"


def _large_inputs(case, fixture_rows):
    """Full-size X on the device (fast generator) with the fixture rows regenerated exactly,
    and the seeded weights."""
    from tests.golden.make_golden import logical_x_rows

    p = C.case_problem(case)
    dtype = getattr(torch, p.dtype)
    g = torch.Generator(device="cuda").manual_seed(7)
    x = torch.randn((p.m, p.k), generator=g, device="cuda", dtype=torch.float32).to(dtype)
    xr = logical_x_rows(case, fixture_rows)
    x[torch.as_tensor(fixture_rows, device="cuda")] = torch.from_numpy(xr.view(np.int16)).view(dtype).cuda()
    w1b, w2b = C.weights(case)
    w1 = torch.from_numpy(w1b.view(np.int16)).view(dtype).cuda()
    w2 = torch.from_numpy(w2b.view(np.int16)).view(dtype).cuda()
    return x.view(p.input_shape), w1, w2, w1b, w2b


@pytest.mark.parametrize("tile", [None, "pair256x256", "cta128x256"])
@pytest.mark.parametrize("case_id", ["cfg4_bf16", "cfg5_bf16"])
def test_full_size_vs_golden_and_oracle(case_id, tile):
    case = C.get_case(case_id)
    fx = np.load(GOLDEN / f"{case_id}.npz")
    p = C.case_problem(case)
    x, w1, w2, w1b, w2b = _large_inputs(case, fx["rows"])
    prepared, y = run(x, w1, w2, down_impl=case["down_impl"], tile=tile)
    got = rows_of(y, fx["rows"])
    assert_close_bits(got, fx["staged_rational"], p.dtype)
    assert_criterion(got, fx["golden"], p.dtype)
    # random rows across the whole M range against the oracle
    rng = np.random.Generator(np.random.PCG64(3))
    rows = np.sort(rng.choice(p.m, size=48, replace=False))
    xs = bits_of(x.reshape(p.m, p.k)[torch.as_tensor(rows, device="cuda")])
    ref = O.ffn(O.from_bits(xs, p.dtype), O.from_bits(w1b, p.dtype), O.from_bits(w2b, p.dtype), p.dtype,
                staged=True, rational=True)
    assert_close_bits(rows_of(y, rows), ref, p.dtype)
    first = bits_of(y)
    prepared.run()
    prepared.check()
    assert np.array_equal(bits_of(y), first), "run-to-run results differ"


def test_pair_placement_map_keeps_results():
    """CTA-pair plans get a measured owner map (a permutation of the pairs); placing the
    tiles in launch order instead, or in a reversed order, gives bit-identical output."""
    m, k, h, n = 4096, 1024, 2048, 512
    g = torch.Generator().manual_seed(11)
    x = torch.randn(m, k, generator=g).bfloat16().cuda()
    w1 = (torch.randn(h, k, generator=g) * k ** -0.5).bfloat16().cuda()
    w2 = (torch.randn(n, h, generator=g) * h ** -0.5).bfloat16().cuda()
    prepared, y = run(x, w1, w2, tile="pair256x256")
    owners = prepared.owner_map()
    pairs = prepared.plan.block_num // 2
    if prepared.plan.block_num == torch.cuda.get_device_properties(0).multi_processor_count:
        assert owners is not None and sorted(owners) == list(range(pairs))
    first = bits_of(y)
    for order in (None, list(range(pairs))[::-1]):
        prepared.set_owner_map(order)
        assert prepared.owner_map() == order
        prepared.run()
        prepared.check()
        assert np.array_equal(bits_of(y), first)
    with pytest.raises(ValueError):
        prepared.set_owner_map([0] * pairs)
    smid = prepared.trace()["smid"]
    assert len(set(smid)) == prepared.plan.block_num


@pytest.mark.parametrize("tile", ["cta128x256", "pair256x256", "cta128x128"])
def test_static_and_dynamic_schedules_agree(tile):
    """Every data-parallel tile is computed whole by one CTA and Stream-K parts keep their
    static split, so the tile order (static, claimed, or static with wave synchronisation)
    cannot change a single bit; repeated launches (epoch bases) agree too."""
    m, k, h, n = 12288, 1024, 4096, 1536
    g = torch.Generator().manual_seed(9)
    x = torch.randn(m, k, generator=g).bfloat16().cuda()
    w1 = (torch.randn(h, k, generator=g) * k ** -0.5).bfloat16().cuda()
    w2 = (torch.randn(n, h, generator=g) * h ** -0.5).bfloat16().cuda()
    outs = []
    for schedule in ("static", "dynamic", "static_synced"):
        for down in ("basic", "streamk"):
            prepared, y = run(x, w1, w2, tile=tile, schedule=schedule, down_impl=down)
            assert prepared.plan.kernel["schedule"] == {"static": 1, "dynamic": 2, "static_synced": 3}[schedule]
            first = bits_of(y)
            for _ in range(3):
                prepared.run()
            prepared.check()
            assert np.array_equal(bits_of(y), first)
            outs.append(first)
    assert all(np.array_equal(o, outs[0]) for o in outs[1:]) or all(
        np.array_equal(outs[i], outs[i % 2]) for i in range(len(outs)))


RAGGED = [
    # (M, K, H, N, dtype)
    (1, 8, 8, 8, torch.bfloat16),
    (16, 64, 128, 128, torch.float16),
    (17, 72, 200, 136, torch.bfloat16),
    (64, 4096, 384, 256, torch.bfloat16),
    (65, 96, 520, 72, torch.float16),
    (129, 136, 264, 264, torch.bfloat16),
    (300, 1000, 1500, 700, torch.bfloat16),
    (1000, 100, 1000, 250, torch.float16),
    (2048, 512, 1024, 384, torch.bfloat16),
]


@pytest.mark.parametrize("shape", RAGGED, ids=lambda s: "x".join(map(str, s[:4])) + str(s[4])[-4:])
@pytest.mark.parametrize("down_impl", ["basic", "streamk"])
@pytest.mark.parametrize("tile", [None, "pair256x256", "cta128x128"])
def test_ragged_shapes_vs_oracle(shape, down_impl, tile):
    m, k, h, n, dtype = shape
    g = torch.Generator().manual_seed(m * 31 + k)
    x = torch.randn(m, k, generator=g).to(dtype)
    w1 = (torch.randn(h, k, generator=g) * k ** -0.5).to(dtype)
    w2 = (torch.randn(n, h, generator=g) * h ** -0.5).to(dtype)
    try:
        _, y = run(x.cuda(), w1.cuda(), w2.cuda(), down_impl=down_impl, tile=tile)
    except NotApplicable:
        pytest.skip("Stream-K not applicable")
    dt = str(dtype).removeprefix("torch.")
    f = lambda t: t.float().numpy()  # noqa: E731
    ref = O.ffn(f(x), f(w1), f(w2), dt, staged=True, rational=True)
    assert_close_bits(bits_of(y), ref, dt)


RAGGED_N512 = [s for s in [
    (1, 8, 8, 8, torch.bfloat16), (16, 64, 128, 128, torch.float16), (17, 72, 200, 136, torch.bfloat16),
    (64, 4096, 384, 256, torch.bfloat16), (65, 96, 520, 72, torch.float16), (129, 136, 264, 264, torch.bfloat16),
    (1000, 100, 1000, 250, torch.float16), (2048, 512, 1024, 200, torch.bfloat16), (300, 1000, 1500, 64, torch.bfloat16),
    (4500, 40, 72, 129, torch.float16), (512, 512, 2048, 512, torch.float16), (200, 128, 640, 384, torch.bfloat16),
    (33, 256, 1000, 300, torch.float16), (300, 64, 1000, 520, torch.bfloat16)]]


@pytest.mark.parametrize("shape", RAGGED_N512, ids=lambda s: "x".join(map(str, s[:4])) + str(s[4])[-4:])
@pytest.mark.parametrize("block_num", [None, 3])
def test_full_load_a_vs_oracle(shape, block_num):
    """Hidden-resident row blocks against the oracle (its H sum runs in 128-column chunks;
    the oracle's in one pass: within the same two-ulp bound), ragged in every dimension,
    one CTA per row block or several row blocks per CTA; 256 < N <= 512 as two Y halves per
    row block; N > 512 is not applicable."""
    m, k, h, n, dtype = shape
    g = torch.Generator().manual_seed(m * 13 + n)
    x = torch.randn(m, k, generator=g).to(dtype)
    w1 = (torch.randn(h, k, generator=g) * k ** -0.5).to(dtype)
    w2 = (torch.randn(n, h, generator=g) * h ** -0.5).to(dtype)
    if n > 512:
        with pytest.raises(NotApplicable):
            prepare_ffn(x.cuda(), w1.cuda(), w2.cuda(), down_impl="full_load_a")
        return
    prepared, y = run(x.cuda(), w1.cuda(), w2.cuda(), down_impl="full_load_a", block_num=block_num)
    assert prepared.plan.kernel["variant"] in (7, 8, 9) and prepared.storage[3].shape[1] == 8
    dt = str(dtype).removeprefix("torch.")
    f = lambda t: t.float().numpy()  # noqa: E731
    ref = O.ffn(f(x), f(w1), f(w2), dt, staged=True, rational=True)
    assert_close_bits(bits_of(y), ref, dt)
    first = bits_of(y)
    prepared.run()
    prepared.check()
    assert np.array_equal(bits_of(y), first)


@pytest.mark.parametrize("case_id", ["cfg1_fp16", "cfg2_fp16", "cfg2_bf16"])
@pytest.mark.parametrize("gelu", ["rational", "erf"])
def test_full_load_a_small_configs_vs_reference_golden(case_id, gelu):
    case = C.get_case(case_id)
    fx = np.load(GOLDEN / f"{case_id}.npz")
    dt = str(fx["dtype"])
    x, w1, w2 = C.make_inputs(case, device="cuda")
    _, y = run(x, w1, w2, down_impl="full_load_a", gelu=gelu)
    got = rows_of(y, fx["rows"])
    assert_criterion(got, fx["golden"], dt)
    if gelu == "rational":
        assert_close_bits(got, fx["staged_rational"], dt)
    else:
        assert_close_bits(got, fx["golden"], dt, floor=4e-3)


@pytest.mark.parametrize("block_num", [1, 3, 37, 148])
def test_block_num_variants(block_num):
    case = C.get_case("cfg2_bf16")
    fx = np.load(GOLDEN / "cfg2_bf16.npz")
    x, w1, w2 = C.make_inputs(case, device="cuda")
    for down in ("basic", "streamk"):
        try:
            _, y = run(x, w1, w2, down_impl=down, block_num=block_num)
        except NotApplicable:
            continue
        got = rows_of(y, fx["rows"])
        assert_close_bits(got, fx["staged_rational"], "bfloat16")


def test_prepared_semantics():
    case = C.get_case("cfg1_fp16")
    x, w1, w2 = C.make_inputs(case, device="cuda")
    prepared = prepare_ffn(x, w1, w2)
    y1 = prepared.run()
    y2 = prepared.run()
    assert y1.data_ptr() == y2.data_ptr()  # one reused output buffer
    assert tuple(y1.shape) == (4, 128, 512)
    assert prepared.preparation["auxiliary_device_interval_ms"] >= 0
    side = torch.cuda.Stream()
    with torch.cuda.stream(side):
        with pytest.raises(RuntimeError, match="preparation stream"):
            prepared.run()
    # new input through run(x): equals a fresh prepare on that input
    x2 = torch.randn_like(x.float()).to(x.dtype)
    y3 = prepared.run(x2).clone()
    ref = prepare_ffn(x2, w1, w2).run()
    assert torch.equal(y3, ref)
    with pytest.raises(ValueError):
        prepare_ffn(x, w1, w2, block_num=10_000)


@pytest.mark.parametrize("case_id,chunks", [("cfg1_fp16", 4), ("cfg2_bf16", 5), ("cfg3_bf16", 2)])
def test_run_host_matches_run(case_id, chunks):
    """Host-to-host path with overlapped copies equals the device path (ragged chunks, padded
    pitches), twice in a row with different inputs."""
    case = C.get_case(case_id)
    p = C.case_problem(case)
    x, w1, w2 = C.make_inputs(case, device="cuda")
    prepared = prepare_ffn(x, w1, w2, down_impl=case["down_impl"])
    xh = x.contiguous().cpu().pin_memory()
    yh = torch.empty(p.output_shape, dtype=x.dtype, pin_memory=True)
    for step in range(2):
        if step:
            xh.copy_((xh.float() * -0.5).to(x.dtype))
        want = prepare_ffn(xh.cuda(), w1, w2, down_impl=case["down_impl"]).run().cpu()
        prepared.run_host(xh, yh, chunks=chunks)
        prepared.check()
        dt = p.dtype
        assert_close_bits(bits_of(yh.reshape(-1, p.n)), bits_of(want.reshape(-1, p.n)), dt)
