"""N > 1 host logic on CPU ranks (gloo, world size 2, 127.0.0.1).

- Distributed SpMV (muda_b200.dist_spmv): the nnz-balanced row partition, the
  rebased local blocks and the x exchange, with the oracle's CPU SpMV standing in
  for the local CUDA product; the ranks' y blocks must reproduce the
  single-device oracle result bit for bit (same per-row fma order).
- RNG weak scaling (muda_b200.partition): the ranks' counter ranges are disjoint
  and contiguous, so their concatenated streams equal one generator's stream.
"""

import os
import socket

import numpy as np
import pytest

import oracle
from muda_b200.dist_spmv import nnz_balanced_bounds, x_block
from muda_b200.partition import rng_rank_offset

WORLD = 2


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(fn, *args):
    import torch.multiprocessing as mp
    port = _free_port()
    mp.start_processes(fn, args=(WORLD, port, *args), nprocs=WORLD, join=True,
                       start_method="spawn")


def _init(rank, world, port):
    import datetime

    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    return dist


def _csr(seed, rows, cols, heavy_rows=()):
    rng = np.random.default_rng(seed)
    k = np.minimum(rng.integers(0, 9, rows), cols)
    for r in heavy_rows:
        k[r] = min(cols, 400)
    ro = np.zeros(rows + 1, np.int64)
    ro[1:] = np.cumsum(k)
    ci = np.concatenate([np.sort(rng.choice(cols, kk, replace=False)) for kk in k]
                        ).astype(np.int32) if ro[-1] else np.zeros(0, np.int32)
    va = rng.uniform(-1, 1, ro[-1]).astype(np.float32)
    x = rng.uniform(-1, 1, cols).astype(np.float32)
    return ro.astype(np.int32), ci, va, x


def _cpu_local(offsets, col_ind, values, x, y, alpha, beta):
    out = oracle.spmv_csr(offsets.numpy(), col_ind.numpy(), values.numpy(), x.numpy(),
                          alpha=alpha, beta=beta, y=y.numpy()[:len(offsets) - 1].copy(),
                          threads=1)
    y[:len(out)] = __import__("torch").from_numpy(out)


def _spmv_worker(rank, world, port, rows, cols, heavy, alpha, beta, overlap=False):
    import torch

    from muda_b200.dist_spmv import DistSpMV
    dist = _init(rank, world, port)
    try:
        ro, ci, va, x = _csr(11, rows, cols, heavy)
        y0 = np.random.default_rng(3).uniform(-1, 1, rows).astype(np.float32)
        d = DistSpMV.from_full(torch, dist, None, torch.from_numpy(ro), torch.from_numpy(ci),
                               torch.from_numpy(va), cols, local_spmv=_cpu_local,
                               overlap=overlap)
        assert d.bounds == nnz_balanced_bounds(ro, world)
        x_local = d.x_slice(torch.from_numpy(x))
        y_local = torch.from_numpy(y0[d.row_begin:d.row_end].copy())
        d.spmv(alpha, x_local, beta, y_local)
        # the gathered x is the full vector on every rank
        assert np.array_equal(d.x_full[:cols].numpy(), x)
        # collect every rank's y block on every rank (pad to the longest block)
        n_max = max(d.bounds[i + 1] - d.bounds[i] for i in range(world))
        pad = torch.zeros(n_max, dtype=torch.float32)
        pad[:d.rows] = y_local
        parts = [torch.zeros(n_max, dtype=torch.float32) for _ in range(world)]
        dist.all_gather(parts, pad)
        y = np.concatenate([parts[i][:d.bounds[i + 1] - d.bounds[i]].numpy()
                            for i in range(world)])
        want = oracle.spmv_csr(ro, ci, va, x, alpha=alpha, beta=beta, y=y0.copy(), threads=1)
        if not overlap:
            assert np.array_equal(y.view(np.uint32), want.view(np.uint32))
        else:
            # each row summed in two parts (own x block, then the rest): within the
            # float32 summation bound of the one-pass product
            _assert_within_sum_bound(ro, ci, va, x, y0, alpha, beta, y)
        # nnz balance: every block within one row's length of nnz / world
        nnz = int(ro[-1])
        longest = int(np.max(np.diff(ro))) if rows else 0
        for i in range(world):
            share = int(ro[d.bounds[i + 1]] - ro[d.bounds[i]])
            assert abs(share - nnz / world) <= longest + 1
        d.close()
    finally:
        dist.destroy_process_group()


def _assert_within_sum_bound(ro, ci, va, x, y0, alpha, beta, y):
    """|y - exact| <= (row length + 3) * 2^-24 * (|alpha| sum |a x| + |beta y0|) per row."""
    rows = len(ro) - 1
    exact = beta * y0.astype(np.float64)
    mag = np.abs(beta * y0.astype(np.float64))
    for r in range(rows):
        s = slice(ro[r], ro[r + 1])
        p = va[s].astype(np.float64) * x[ci[s]].astype(np.float64)
        exact[r] += alpha * p.sum()
        mag[r] += abs(alpha) * np.abs(p).sum()
    bound = (np.diff(ro) + 3) * 2.0 ** -24 * mag + 1e-30
    assert np.all(np.abs(y.astype(np.float64) - exact) <= bound)


def _rng_worker(rank, world, port, n, seed):
    import torch
    dist = _init(rank, world, port)
    try:
        off = rng_rank_offset(rank, n)
        assert off % 4 == 0
        mine, end = oracle.generate_uint(seed, off, 2 * n)
        assert end == off + 2 * n
        parts = [torch.zeros(2 * n, dtype=torch.int64) for _ in range(world)]
        dist.all_gather(parts, torch.from_numpy(mine.astype(np.int64)))
        got = np.concatenate([p.numpy() for p in parts]).astype(np.uint32)
        want, _ = oracle.generate_uint(seed, 0, 2 * n * world)
        assert np.array_equal(got, want)
        # the uniform and normal blocks of this rank are the reference's calls at
        # its offset: uniform at off, normal right after
        u, after = oracle.generate_uniform(seed, off, n)
        z, _ = oracle.generate_normal(seed, after, n, 0.0, 1.0)
        assert after == off + n and np.isfinite(z).all() and (u > 0).all() and (u <= 1).all()
    finally:
        dist.destroy_process_group()


def test_nnz_balanced_bounds_edges():
    ro = np.array([0, 2, 4, 6, 8], np.int64)
    assert nnz_balanced_bounds(ro, 2) == [0, 2, 4]
    assert nnz_balanced_bounds(ro, 1) == [0, 4]
    # one row outweighs everything: later blocks may be empty, never negative
    ro = np.array([0, 1000, 1001, 1002], np.int64)
    b = nnz_balanced_bounds(ro, 4)
    assert b[0] == 0 and b[-1] == 3 and all(b[i] <= b[i + 1] for i in range(4))
    # more parts than rows, and an empty matrix
    assert nnz_balanced_bounds(np.array([0, 3], np.int64), 4)[-1] == 1
    assert nnz_balanced_bounds(np.zeros(6, np.int64), 3) == [0, 0, 0, 5]
    assert x_block(10, 4) == 3 and x_block(8, 4) == 2
    with pytest.raises(ValueError):
        nnz_balanced_bounds(ro, 0)


@pytest.mark.parametrize("rows,cols,heavy,alpha,beta", [(1000, 777, (), 1.0, 0.0),
                                                        (513, 2049, (0, 7), 0.5, -2.0),
                                                        (3, 5, (), 1.0, 1.0)])
def test_dist_spmv_two_gloo_ranks(rows, cols, heavy, alpha, beta):
    _run(_spmv_worker, rows, cols, heavy, alpha, beta)


@pytest.mark.parametrize("rows,cols,heavy", [(1000, 777, ()), (513, 2049, (0, 7)), (3, 5, ())])
def test_dist_spmv_overlap_two_gloo_ranks(rows, cols, heavy):
    """The overlapped step (own x block first, the rest after the exchange)."""
    _run(_spmv_worker, rows, cols, heavy, 0.5, -2.0, True)


def test_split_by_columns_keeps_every_entry_in_row_order():
    import torch

    from muda_b200.dist_spmv import split_by_columns
    ro, ci, va, _ = _csr(5, 300, 500, (4,))
    for base in (0, 1):
        for lo, hi in ((0, 500), (100, 250), (499, 500), (300, 300)):
            own, rest = split_by_columns(torch, torch.from_numpy(ro + base),
                                         torch.from_numpy(ci + base), torch.from_numpy(va),
                                         base, lo, hi)
            o_ro, o_ci, o_va = (t.numpy() for t in own)
            r_ro, r_ci, r_va = (t.numpy() for t in rest)
            assert o_ro[0] == base and r_ro[0] == base
            for r in range(300):
                s = slice(ro[r], ro[r + 1])
                c, v = ci[s], va[s]
                m = (c >= lo) & (c < hi)
                so = slice(o_ro[r] - base, o_ro[r + 1] - base)
                sr = slice(r_ro[r] - base, r_ro[r + 1] - base)
                assert np.array_equal(o_ci[so] - base + lo, c[m])
                assert np.array_equal(o_va[so], v[m])
                assert np.array_equal(r_ci[sr] - base, c[~m])
                assert np.array_equal(r_va[sr], v[~m])


def test_rng_weak_scaling_partition_two_gloo_ranks():
    _run(_rng_worker, 4099 * 4, 1234)


def test_dist_spmv_exchange_arguments():
    """The exchange is "nccl" or "peer"; the peer exchange is the CUDA path only, so
    a pluggable CPU product with it is refused before anything is allocated."""
    import torch

    from muda_b200.dist_spmv import DistSpMV
    offsets = torch.tensor([0, 1, 2], dtype=torch.int32)
    cols = torch.tensor([0, 1], dtype=torch.int32)
    vals = torch.tensor([1.0, 2.0])
    common = dict(offsets=offsets, col_ind=cols, values=vals, row_begin=0, row_end=2, cols=2,
                  local_spmv=lambda *a: None)
    with pytest.raises(ValueError, match="unknown exchange"):
        DistSpMV(torch, None, None, exchange="nvshmem", **common)
    with pytest.raises(ValueError, match="CUDA path only"):
        DistSpMV(torch, None, None, exchange="peer", **common)
    d = DistSpMV(torch, None, None, exchange="nccl", **common)
    x = torch.tensor([3.0, 4.0])
    d.gather_x(x)
    assert torch.equal(d.x_full[:2], x)
