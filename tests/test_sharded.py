"""Host logic of the multi-GPU path on CPU ``gloo`` ranks (no GPU).

Each rank computes its H-slice partial of the FFN with the oracle's arithmetic (fp32) and
the ranks combine them with the same ``combine_partials`` / ``chunk_rows`` /
``scattered_rows`` the GPU ``TensorParallelFFN`` uses; the assembled result must equal the
single-device computation.  The M-shard row split is checked the same way.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from ffn_optim_b200.sharded import band_order, chunk_rows, combine_partials, h_slice, m_slices, scattered_rows
from oracle import ffn_oracle as O


def test_h_slice_partition():
    for h in (8, 100, 1000, 16384, 28672, 65535):
        for world in (1, 2, 3, 4, 8):
            cuts = [h_slice(h, r, world) for r in range(world)]
            assert cuts[0][0] == 0 and cuts[-1][1] == h
            for (a, b), (c, d) in zip(cuts, cuts[1:]):
                assert b == c and b % 8 == 0
            sizes = [b - a for a, b in cuts]
            assert max(sizes) - min(sizes) < 16


def test_m_slices_and_chunks():
    for m in (1, 7, 6993, 65536):
        for world in (1, 2, 3, 8):
            s = m_slices(m, world)
            assert s[0][0] == 0 and s[-1][1] == m and all(b == c for (_, b), (c, _) in zip(s, s[1:]))
    ch = chunk_rows(65536, 8, 4)
    assert ch[0] == (0, 16384) and ch[-1][1] == 65536
    with pytest.raises(ValueError):
        chunk_rows(6993, 2, 4)
    rows = sorted(r for rank in range(8) for r in scattered_rows(ch, rank, 8))
    assert rows == list(range(65536))


def test_tp_dp_layout():
    from ffn_optim_b200.sharded import tp_dp_groups, tp_dp_rows

    assert tp_dp_groups(8, 2) == [[0, 1], [2, 3], [4, 5], [6, 7]]
    assert tp_dp_groups(8, 8) == [list(range(8))]
    for bad in ((8, 3), (4, 1), (4, 8)):
        with pytest.raises(ValueError):
            tp_dp_groups(*bad)
    m = 65536
    for world, tp in ((8, 2), (8, 4), (4, 2), (2, 2)):
        rows = [tp_dp_rows(m, world, tp, r) for r in range(world)]
        assert rows[0][0] == 0 and rows[-1][1] == m
        assert all(a[1] == b[0] for a, b in zip(rows, rows[1:]))  # contiguous, disjoint, in rank order
        assert len({hi - lo for lo, hi in rows}) == 1
    with pytest.raises(ValueError):
        tp_dp_rows(1001, 4, 2, 0)


def test_band_order_puts_own_band_last():
    for world in (2, 3, 8):
        for rank in range(world):
            order = band_order(world, rank)
            assert sorted(order) == list(range(world)) and order[-1] == rank
            # every other rank's band comes before this rank's own band
            for other in range(world):
                if other != rank:
                    assert band_order(world, other).index(rank) < world - 1


def _rs_protocol(world, tiles, rng, flush_before_own=True):
    """Model of the fused reduce-scatter's down phase on `world` ranks (one warp each): rank r
    visits the bands in ``band_order``; a pushed tile's count is released one tile late (when
    the next push is issued) and flushed before an own-band tile and at the end; an own-band
    tile waits for every other rank's count of that tile.  Ranks step in a random order;
    returns True when every rank finishes, False when all unfinished ranks are blocked."""
    work = {r: [(b, j) for b in band_order(world, r) for j in range(tiles)] for r in range(world)}
    pos = {r: 0 for r in range(world)}
    pending = {r: None for r in range(world)}
    released = set()  # (sender, band, tile)
    while True:
        live = [r for r in range(world) if pos[r] <= len(work[r])]
        if not live:
            return True
        progressed = False
        for r in rng.permutation(live):
            r = int(r)
            if pos[r] == len(work[r]):  # end of the work list: flush
                if pending[r] is not None:
                    released.add((r,) + pending[r])
                    pending[r] = None
                pos[r] += 1
                progressed = True
                continue
            b, j = work[r][pos[r]]
            if b != r:  # push: release the previous pushed tile, keep this one pending
                if pending[r] is not None:
                    released.add((r,) + pending[r])
                pending[r] = (b, j)
                pos[r] += 1
                progressed = True
            else:
                if flush_before_own and pending[r] is not None:
                    released.add((r,) + pending[r])
                    pending[r] = None
                    progressed = True
                if all((o, r, j) in released for o in range(world) if o != r):
                    pos[r] += 1
                    progressed = True
        if not progressed:
            return False


@pytest.mark.parametrize("world", [2, 3, 4, 8])
def test_deferred_push_release_is_live(world):
    """The one-tile-late release of pushed partials cannot deadlock: with the flush before
    own-band tiles every random interleaving finishes; without it the model finds the
    deadlock (a rank's last push stays pending while it waits on the others)."""
    rng = np.random.Generator(np.random.PCG64(world))
    for tiles in (1, 2, 5):
        for _ in range(20):
            assert _rs_protocol(world, tiles, rng)
    assert not all(_rs_protocol(world, tiles, rng, flush_before_own=False) for _ in range(20))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _problem(seed=0, m=48, k=40, h=200, n=24):
    rng = np.random.Generator(np.random.PCG64(seed))
    x = O.round_to(rng.standard_normal((m, k), dtype=np.float32), "bfloat16")
    w1 = O.round_to(rng.standard_normal((h, k), dtype=np.float32) * np.float32(k ** -0.5), "bfloat16")
    w2 = O.round_to(rng.standard_normal((n, h), dtype=np.float32) * np.float32(h ** -0.5), "bfloat16")
    return x, w1, w2


def _partial(x, w1, w2, lo, hi):
    hidden = O.round_to(O.gelu_rational(x @ w1[lo:hi].T), "bfloat16")
    return hidden @ w2[:, lo:hi].T


def _worker(rank, world, port, mode, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        x, w1, w2 = _problem()
        lo, hi = h_slice(w1.shape[0], rank, world)
        partial = torch.from_numpy(np.ascontiguousarray(_partial(x, w1, w2, lo, hi)))
        if mode == "reduce_scatter":
            chunks = chunk_rows(x.shape[0], world, 3)
            outs, works = [], []
            for a, b in chunks:
                out = torch.empty(((b - a) // world, partial.shape[1]))
                works.append(combine_partials(partial[a:b].contiguous(), out, mode, async_op=True))
                outs.append(out)
            for w in works:
                w.wait()
            rows = scattered_rows(chunks, rank, world)
            np.save(os.path.join(out_dir, f"r{rank}.npy"), torch.cat(outs).numpy())
            np.save(os.path.join(out_dir, f"i{rank}.npy"), np.array(rows))
        else:
            combine_partials(partial, None, mode)
            np.save(os.path.join(out_dir, f"r{rank}.npy"), partial.numpy())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
@pytest.mark.parametrize("mode", ["reduce_scatter", "all_reduce"])
def test_tensor_parallel_composition_gloo(world, mode, tmp_path):
    mp.spawn(_worker, args=(world, _free_port(), mode, str(tmp_path)), nprocs=world, join=True)
    x, w1, w2 = _problem()
    full = _partial(x, w1, w2, 0, w1.shape[0])
    if mode == "reduce_scatter":
        got = np.zeros_like(full)
        seen = []
        for r in range(world):
            rows = np.load(tmp_path / f"i{r}.npy")
            got[rows] = np.load(tmp_path / f"r{r}.npy")
            seen.extend(rows.tolist())
        assert sorted(seen) == list(range(full.shape[0]))
    else:
        got = np.load(tmp_path / "r0.npy")
        for r in range(1, world):
            assert np.array_equal(np.load(tmp_path / f"r{r}.npy"), got)
    # the sum of H-slice partials is the whole FFN (fp32 summation order only)
    assert np.allclose(got, full, rtol=1e-5, atol=1e-5 * np.abs(full).max())
    assert (O.to_bits(got, "bfloat16") == O.to_bits(full, "bfloat16")).mean() > 0.99
