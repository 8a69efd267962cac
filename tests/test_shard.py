"""Row sharding of the packed matvec, on CPU: the row split (efg_shard_rows) and the
exchange pattern of efg_matvec_sharded (in-place all-gather for an even split, one
broadcast per rank otherwise) run by world_size-2 gloo ranks over the CPU oracle's
per-shard matvecs. The assembled y must be bit-identical to the unsharded matvec (each
row's dot is computed by exactly one rank, in the same order)."""
from __future__ import annotations

import ctypes as C
import os
import socket

import numpy as np
import pytest

import edgeforge_b200 as efg
from oracle.oracle import Q4_0, Q8_0


def test_shard_rows_is_chunk_begin():
    for rows in (0, 1, 7, 1000, 1001, 131072, 32000):
        for n in (1, 2, 3, 4, 8):
            end = 0
            for r in range(n):
                b, c = efg.shard_rows(rows, n, r)
                assert b == rows * r // n and b + c == rows * (r + 1) // n  # ThreadPool::chunk_begin
                assert b == end
                end = b + c
            assert end == rows


def test_shard_rows_rejects_bad_rank():
    for n, r in ((0, 0), (2, 2), (2, -1)):
        with pytest.raises(efg.EdgeForgeError):
            efg.shard_rows(10, n, r)


def test_sharded_rejects_null_comm():
    lib = efg.load()
    assert lib.efg_matvec_sharded(Q4_0, None, None, None, 10, 64, None, None) == 1
    assert "null communicator" in lib.efg_last_error().decode()
    assert lib.efg_comm_destroy(None) == 0


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, qt, rows, cols, out_dir):
    import torch
    import torch.distributed as dist

    from oracle.oracle import Oracle, row_bytes

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    o = Oracle()
    rng = np.random.default_rng(7)  # every rank builds the same matrix and x
    W = o.quantize_rows(qt, (0.02 * rng.standard_normal((rows, cols))).astype(np.float32), threads=1)
    x = rng.standard_normal(cols).astype(np.float32)
    b, c = efg.shard_rows(rows, world, rank)
    y = torch.zeros(rows, dtype=torch.float32)
    if c:
        rb = row_bytes(qt, cols)
        shard = W.reshape(rows, rb)[b:b + c]
        y[b:b + c] = torch.from_numpy(o.matvec(qt, shard, x, c))
    if rows % world == 0:  # the all-gather case
        parts = [torch.empty(rows // world) for _ in range(world)]
        dist.all_gather(parts, y[b:b + c].clone())
        y = torch.cat(parts)
    else:  # one broadcast per rank, each from the rank that owns the slice
        for r in range(world):
            rb_, rc_ = efg.shard_rows(rows, world, r)
            if rc_:
                sl = y[rb_:rb_ + rc_].clone()
                dist.broadcast(sl, src=r)
                y[rb_:rb_ + rc_] = sl
    np.save(os.path.join(out_dir, f"y{rank}.npy"), y.numpy())
    if rank == 0:
        np.save(os.path.join(out_dir, "full.npy"), o.matvec(qt, W, x, rows))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("qt,rows,cols", [(Q4_0, 1000, 256), (Q4_0, 1001, 256), (Q8_0, 333, 128)])
def test_two_gloo_ranks_assemble_full_y(tmp_path, qt, rows, cols):
    import torch.multiprocessing as mp

    mp.start_processes(_rank_main, args=(2, _free_port(), qt, rows, cols, str(tmp_path)), nprocs=2, join=True,
                       start_method="spawn")
    full = np.load(tmp_path / "full.npy")
    for r in range(2):
        np.testing.assert_array_equal(np.load(tmp_path / f"y{r}.npy"), full)


def _local_pair(shard, offset):
    """One shard's candidate under kern::argmax's rule (src/kernels.cpp:105-111): the largest
    non-NaN value with the lowest index; (None, -2) when the shard starts the vector with a
    NaN; (None, -1) when it has no non-NaN value. Mirrors argmax_local_kernel."""
    if offset == 0 and shard.size and np.isnan(shard[0]):
        return (0.0, -2)
    ok = ~np.isnan(shard)
    if not ok.any():
        return (0.0, -1)
    best = shard[ok].max()
    return (float(best), offset + int(np.nonzero(shard == best)[0][0]))


def _combine(pairs):
    """argmax_combine_kernel: shards in index order, strictly greater wins."""
    idx, best = -1, 0.0
    for v, i in pairs:
        if i == -2:
            return 0
        if i >= 0 and (idx < 0 or v > best):
            idx, best = i, v
    return max(idx, 0)


def _argmax_rank(rank, world, port, cases, out_dir):
    import torch
    import torch.distributed as dist

    from oracle.oracle import Oracle

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    o = Oracle()
    got = []
    for v in cases:
        b, c = efg.shard_rows(v.size, world, rank)
        mine = torch.tensor(_local_pair(v[b:b + c], b), dtype=torch.float64)
        parts = [torch.empty(2, dtype=torch.float64) for _ in range(world)]
        dist.all_gather(parts, mine)
        got.append((_combine([(float(t[0]), int(t[1])) for t in parts]), o.argmax(v)))
    np.save(os.path.join(out_dir, f"argmax{rank}.npy"), np.array(got))
    dist.barrier()
    dist.destroy_process_group()


def test_two_gloo_ranks_distributed_argmax(tmp_path):
    """The row-sharded argmax (efg_lm_head_argmax_sharded) decomposes kern::argmax exactly:
    per-shard pairs combined in rank order equal the reference's argmax of the whole vector
    on ties across shards, NaN at index 0, NaN elsewhere, an all-NaN shard and maxima at a
    shard edge."""
    import torch.multiprocessing as mp

    rng = np.random.default_rng(3)
    v = rng.standard_normal(1001).astype(np.float32)
    tie = v.copy()
    tie[[100, 900]] = 9.0  # the same maximum in both shards
    nan0 = v.copy()
    nan0[0] = np.nan
    nans = v.copy()
    nans[::7] = np.nan
    allnan_b = v.copy()
    allnan_b[500:] = np.nan  # the second shard holds no number
    edge = v.copy()
    edge[500] = 7.0  # first element of shard 1
    edge2 = v.copy()
    edge2[499] = 7.0  # last element of shard 0
    neg = np.full(16, -np.inf, np.float32)
    cases = [v, tie, nan0, nans, allnan_b, edge, edge2, neg]
    mp.start_processes(_argmax_rank, args=(2, _free_port(), cases, str(tmp_path)), nprocs=2, join=True,
                       start_method="spawn")
    for r in range(2):
        got = np.load(tmp_path / f"argmax{r}.npy")
        np.testing.assert_array_equal(got[:, 0], got[:, 1])


def test_comm_symbols_present():
    lib = efg.load()
    for name in ("efg_comm_unique_id", "efg_comm_init", "efg_comm_destroy", "efg_matvec_sharded", "efg_shard_rows",
                 "efg_argmax", "efg_lm_head_argmax_sharded"):
        assert isinstance(getattr(lib, name), C._CFuncPtr)
