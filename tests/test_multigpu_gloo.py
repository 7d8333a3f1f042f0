"""The multi-rank path on CPU: row sharding, global-index seeding, max-over-ranks
timing, and host-side failure detection, with world_size-2 gloo process groups.

The data path has no collective: each rank computes its own contiguous row block
(runner.shard_range) from inputs keyed by global element index, so the shards
concatenated equal the single-rank result bit for bit. The only collectives are
the ones bench.py uses around the timed region (barrier, MAX all-reduce of the
elapsed time). Failure detection is exercised on the host: a rank that exits
without joining makes the survivor's monitored barrier fail within its timeout.
"""
from __future__ import annotations

import datetime
import multiprocessing as mp
import os
import socket

import numpy as np
import pytest

import oracle
import runner

DIMS = dict(dim=256, inter=384, nq=4, nkv=2, hd=64, period=97)


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def keyed_normal(seed: int, start: int, count: int) -> np.ndarray:
    """N(0,1) samples that depend only on (seed, global index): SplitMix64 + Box-Muller."""
    i = np.arange(start, start + count, dtype=np.uint64)
    with np.errstate(over="ignore"):
        z = i + np.uint64(seed) * np.uint64(0xD1B54A32D192ED03) + np.uint64(0x9E3779B97F4A7C15)
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        z = z ^ (z >> np.uint64(31))
    u1 = ((z >> np.uint64(40)).astype(np.float64) + 1.0) / 16777217.0
    u2 = (z & np.uint64(0xFFFFFF)).astype(np.float64) / 16777216.0
    return (np.sqrt(-2.0 * np.log(u1)) * np.cos(2 * np.pi * u2)).astype(np.float32)


def shard_chain(r0: int, r1: int) -> np.ndarray:
    """The layer chain (oracle) on global rows [r0, r1); returns the concatenated outputs."""
    d = DIMS
    n = r1 - r0
    D, I, hd = d["dim"], d["inter"], d["hd"]
    rows = lambda seed, width: keyed_normal(seed, r0 * width, n * width).reshape(n, width)  # noqa
    x, da, df = rows(1, D), rows(2, D), rows(3, D)
    q, k, gu = rows(4, d["nq"] * hd), rows(5, d["nkv"] * hd), rows(6, 2 * I)
    w_in = 1 + 0.02 * keyed_normal(7, 0, D)
    w_post = 1 + 0.02 * keyed_normal(8, 0, D)
    wq, wk = 1 + 0.02 * keyed_normal(9, 0, hd), 1 + 0.02 * keyed_normal(10, 0, hd)
    ct, st = oracle.compute_rope_neox(np.arange(d["period"]), hd, 1e6)
    pos = np.arange(r0, r1) % d["period"]
    c_rows, s_rows = np.ascontiguousarray(ct[pos]), np.ascontiguousarray(st[pos])
    y = np.empty_like(x)
    P = oracle.ptr
    oracle.load().oracle_layer_chain_f32(P(x), P(da), P(df), P(y), P(q), P(k), P(gu), P(w_in),
                                         P(w_post), P(wq), P(wk), P(c_rows), P(s_rows), n, D,
                                         d["nq"], d["nkv"], hd, I, 1e-6)
    return np.concatenate([x, y, q, k, gu[:, :I]], axis=1)


def _worker(rank: int, world: int, port: int, n_rows: int, outdir: str, mode: str) -> None:
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=30))
    if mode == "shard":
        r0, r1 = runner.shard_range(n_rows, world, rank)
        np.save(os.path.join(outdir, f"rank{rank}.npy"), shard_chain(r0, r1))
        t = torch.tensor([float(rank + 1)], dtype=torch.float64)  # stand-in elapsed time
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        with open(os.path.join(outdir, f"max{rank}.txt"), "w") as f:
            f.write(str(t.item()))
        dist.barrier()
        dist.destroy_process_group()
    elif mode == "fail":
        if rank == 1:
            os._exit(3)  # leaves between steps: nothing of it is in flight
        try:
            dist.monitored_barrier(timeout=datetime.timedelta(seconds=4))
            msg = "no error"
        except RuntimeError as e:
            msg = f"error: {e}"
        with open(os.path.join(outdir, "fail0.txt"), "w") as f:
            f.write(msg)
        os._exit(0)


def _run(world: int, n_rows: int, outdir: str, mode: str) -> list[int]:
    ctx = mp.get_context("spawn")
    port = free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, n_rows, outdir, mode))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    codes = []
    for p in procs:
        if p.is_alive():
            p.kill()
            p.join()
        codes.append(p.exitcode)
    return codes


def test_shard_range_partitions_rows():
    for n in (0, 1, 7, 64, 2 ** 21 + 3):
        for world in (1, 2, 3, 4, 8):
            parts = [runner.shard_range(n, world, r) for r in range(world)]
            assert parts[0][0] == 0 and parts[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(parts, parts[1:]))
            sizes = [b - a for a, b in parts]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        runner.shard_range(10, 2, 2)


def test_keyed_inputs_do_not_depend_on_the_split():
    full = keyed_normal(5, 0, 1000)
    assert np.array_equal(np.concatenate([keyed_normal(5, 0, 400), keyed_normal(5, 400, 600)]), full)
    assert abs(full.mean()) < 0.1 and abs(full.std() - 1) < 0.1


def test_two_rank_shards_equal_single_rank(tmp_path):
    n = 301
    codes = _run(2, n, str(tmp_path), "shard")
    assert codes == [0, 0]
    got = np.concatenate([np.load(tmp_path / "rank0.npy"), np.load(tmp_path / "rank1.npy")])
    assert np.array_equal(got, shard_chain(0, n))
    assert (tmp_path / "max0.txt").read_text() == "2.0" == (tmp_path / "max1.txt").read_text()


def test_rank_that_never_joins_is_detected(tmp_path):
    codes = _run(2, 8, str(tmp_path), "fail")
    assert codes[1] == 3
    msg = (tmp_path / "fail0.txt").read_text()
    assert msg.startswith("error") and "1" in msg
