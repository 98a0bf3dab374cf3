"""Multi-GPU paths against the CPU oracle (skipped with fewer than 2 GPUs).

At world size 2 and at every GPU of the box (``torch.cuda.device_count()``), one process per
GPU over NCCL: H-sharded tensor parallelism with the reduce-scatter fused into the kernel
(fp32 partials, the default; fp32 rounded to 24 bits; input-dtype partials), H-sharded with an NCCL
reduce-scatter, M-sharded, and (4 GPUs or more) pairs of GPUs running the fused
reduce-scatter on M slices.  Every rank's output rows are checked against the oracle
(``oracle/ffn_oracle.py``, the numpy restatement of the reference's ``ffn_torch``) on the
same inputs: the reference criterion with the max-abs bound (``compare(strict=True)``)
against the exact-erf golden for every variant, and the single-GPU bound -- two output ulps
+ 1e-3*max|golden| against the golden of the kernel's arithmetic (rational GELU, staged
hidden) -- for the variants that sum unrounded or 24-bit partials (fp32 and fp24
reduce-scatter, M-shard).
The variants that round each rank's partial to bf16 before the cross-GPU sum get a floor of
4e-3*max|golden| instead (up to P-1 extra roundings).
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

SHAPE = (4096, 1024, 4096, 1024)  # M, K, H, N: M divisible by 8 ranks x 128-row tiles


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs():
    m, k, h, n = SHAPE
    g = torch.Generator().manual_seed(11)
    x = torch.randn(m, k, generator=g).bfloat16()
    w1 = (torch.randn(h, k, generator=g) * k ** -0.5).bfloat16()
    w2 = (torch.randn(n, h, generator=g) * h ** -0.5).bfloat16()
    return x, w1, w2


def _worker(rank, world, port, out_dir):
    from datetime import timedelta

    import torch.distributed as dist

    from ffn_optim_b200.sharded import FusedTensorParallelFFN, RowShardedFFN, TensorParallelFFN, TpDpFusedFFN

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
    try:
        x, w1, w2 = (t.to(dev) for t in _inputs())
        out = {}
        tp = TensorParallelFFN(x, w1, w2, chunks=2)
        out["nccl"] = tp.run().float().cpu().numpy()
        tp.check()
        out["nccl_rows"] = np.array(tp.local_rows())
        for partial in ("fp32", "fp24", "input"):
            fused = FusedTensorParallelFFN(x, w1, w2, partial=partial)
            first = None
            for i in range(3):  # repeated launches exercise both staging parities
                y = fused.run()
                fused.check()
                if i == 0:
                    first = y.clone()
            out[f"fused_{partial}"] = y.float().cpu().numpy()
            out[f"fused_{partial}_rows"] = np.array(fused.local_rows())
            out[f"fused_{partial}_repeat_equal"] = np.array(bool(torch.equal(first, y)))
            fused.close()
        ms = RowShardedFFN(x, w1, w2)
        out["m"] = ms.run().float().cpu().numpy()
        ms.check()
        out["m_rows"] = np.arange(ms.lo, ms.hi)
        if world >= 4:  # pairs of GPUs with the fused reduce-scatter, M split over the pairs
            hy = TpDpFusedFFN(x, w1, w2, tp=2)
            for _ in range(2):
                y = hy.run()
                hy.check()
            out["tp2"] = y.float().cpu().numpy()
            out["tp2_rows"] = np.array(hy.local_rows())
            hy.close()
        np.savez(os.path.join(out_dir, f"r{rank}.npz"), **out)
        dist.barrier()
    finally:
        dist.destroy_process_group()


def _oracle():
    from oracle import ffn_oracle as O

    x, w1, w2 = (t.float().numpy() for t in _inputs())
    staged = O.from_bits(O.ffn(x, w1, w2, "bfloat16", staged=True, rational=True), "bfloat16")
    golden = O.from_bits(O.ffn(x, w1, w2, "bfloat16"), "bfloat16")
    return staged, golden


def _check(what, got, staged, golden, floor):
    from ffn_optim_b200 import compare

    r = compare(torch.from_numpy(got), torch.from_numpy(golden), strict=True)
    assert r["passed"], (what, r)
    bound = 2.0 ** -6 * np.abs(staged) + floor * np.abs(staged).max()
    excess = np.abs(got - staged) - bound
    assert np.all(excess <= 0), (what, float(excess.max()))


def _worlds():
    n = torch.cuda.device_count()
    return sorted({2, min(n, 8)}) if n >= 2 else [2]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("world", _worlds())
def test_sharded_variants_vs_oracle(tmp_path, world):
    mp.spawn(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    staged, golden = _oracle()
    keys = ("nccl", "fused_fp32", "fused_fp24", "fused_input", "m") + (("tp2",) if world >= 4 else ())
    seen = {k: np.zeros(SHAPE[0], dtype=bool) for k in keys}
    for r in range(world):
        d = np.load(tmp_path / f"r{r}.npz")
        for key, floor in (("fused_fp32", 1e-3), ("fused_fp24", 1e-3), ("m", 1e-3), ("fused_input", 4e-3),
                           ("nccl", 4e-3), ("tp2", 1e-3)):
            if key not in keys:
                continue
            rows = d[f"{key}_rows"]
            _check(f"{key} rank {r} of {world}", d[key], staged[rows], golden[rows], floor)
            seen[key][rows] = True
        for partial in ("fp32", "fp24", "input"):
            assert bool(d[f"fused_{partial}_repeat_equal"]), f"fused {partial}: run-to-run results differ"
    for key, mask in seen.items():
        assert mask.all(), f"{key}: rows not covered by any rank"


def _dead_rank_worker(rank, world, port, out_dir):
    """Rank 1 leaves between steps (launches nothing for step 2, no kernel or collective in
    flight); rank 0's band owners wait for partials that never come, their bounded wait runs
    out, the kernel reports a peer timeout and returns; the ranks meet again on the host,
    reset together and run a correct step."""
    from datetime import timedelta

    import torch.distributed as dist

    from ffn_optim_b200.sharded import FusedTensorParallelFFN

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
    try:
        x, w1, w2 = (t.to(dev) for t in _inputs())
        fused = FusedTensorParallelFFN(x, w1, w2)
        fused.prepared.set_wait_limit(0.5)
        good = fused.run().clone()
        fused.check()
        dist.barrier()
        status = [0, 0, 0, 0]
        if rank == 0:
            fused.run()
            status = fused.prepared.status()  # synchronises: the kernel has returned
        dist.barrier()
        fused.prepared.reset()  # every rank clears its counts and restarts its epoch
        torch.cuda.synchronize()
        dist.barrier()
        again = fused.run().clone()
        fused.check()
        np.savez(os.path.join(out_dir, f"dead{rank}.npz"), status=np.array(status),
                 same=bool(torch.equal(good, again)))
        fused.close()
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_fused_reduce_scatter_detects_missing_rank(tmp_path):
    mp.spawn(_dead_rank_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True)
    d0 = np.load(tmp_path / "dead0.npz")
    assert int(d0["status"][0]) == 4, d0["status"]  # FFN_B200_KERNEL_PEER_TIMEOUT
    for r in range(2):
        assert bool(np.load(tmp_path / f"dead{r}.npz")["same"])
