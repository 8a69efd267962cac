"""efg_matvec_sharded on the GPU: one rank (the NCCL communicator of a single GPU), and
two to four ranks, one process per GPU, when the machine has them. Each rank quantizes
the same seeded matrix on its own GPU (bit-exact quantizer), keeps its row slice, and the
gathered y must agree with the oracle (|y - exact| / sum|w x| <= 1e-5 per row) and be
identical on every rank."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest

import edgeforge_b200 as efg
from edgeforge_b200 import QType

pytestmark = pytest.mark.gpu
TOL = 1e-5


def _make(torch, qt, rows, cols, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    X = torch.randn(rows, cols, generator=g, device="cuda") * 0.02
    rb = cols // 32 * (18 if qt == QType.Q4_0 else 34)
    W = torch.empty(rows * rb, dtype=torch.uint8, device="cuda")
    efg.quantize_rows(qt, X, rows, cols, W, True)
    x = torch.randn(cols, generator=g, device="cuda")
    return W.view(rows, rb), x


def _check(oracle, qt, W, x, y, rows):
    from conftest import rel_dot_errors

    err = rel_dot_errors(oracle, qt, W.cpu().numpy(), x.cpu().numpy(), rows, y.cpu().numpy())
    assert err.max() <= TOL, err.max()


def test_single_rank(cuda, oracle):
    import torch

    comm = efg.Comm(efg.Comm.unique_id(), 1, 0)
    try:
        for qt, rows, cols in ((QType.Q4_0, 5632, 2048), (QType.Q8_0, 1001, 512)):
            W, x = _make(torch, qt, rows, cols, 3)
            y = torch.full((rows,), float("nan"), device="cuda")
            efg.matvec_sharded(qt, y, W, x, rows, cols, comm)
            ref = torch.empty(rows, device="cuda")
            efg.matvec(qt, ref, W, x, rows, cols)
            torch.cuda.synchronize()
            assert torch.equal(y, ref)
            _check(oracle, qt, W, x, y, rows)
        with pytest.raises(efg.EdgeForgeError, match="divisible by 32"):
            efg.matvec_sharded(QType.Q4_0, y, W, x, rows, 30, comm)
    finally:
        comm.close()
    assert efg.device_error() == 0


def _rmsnorm_host(x, w, eps):
    """h = w * (x * inv), inv = float(1 / sqrt(mean(x^2) + eps)) with the sum in double
    (src/kernels.cpp:69-75)."""
    xd = x.astype(np.float64)
    inv = np.float32(1.0 / np.sqrt((xd * xd).sum() / x.size + eps))
    return (w * (x * inv)).astype(np.float32)


def test_argmax_rule(cuda, oracle):
    """efg_argmax against kern::argmax: ties keep the lower index, NaN never wins except at
    index 0, all-NaN and -inf vectors, unaligned starts, n = 0."""
    import torch

    rng = np.random.default_rng(9)
    v = rng.standard_normal(32000).astype(np.float32)
    cases = [v]
    t = v.copy(); t[[5, 31000]] = 50.0; cases.append(t)
    t = v.copy(); t[0] = np.nan; cases.append(t)
    t = v.copy(); t[::3] = np.nan; cases.append(t)
    cases.append(np.full(1000, np.nan, np.float32))
    cases.append(np.full(37, -np.inf, np.float32))
    t = v[:1001].copy(); t[1000] = 99.0; cases.append(t)
    for c in cases:
        got = efg.argmax(torch.from_numpy(c).cuda())
        assert int(got.item()) == oracle.argmax(c)
    buf = torch.from_numpy(v).cuda()
    assert int(efg.argmax(buf[1:1001]).item()) == oracle.argmax(v[1:1001])  # 4-byte offset: scalar path
    assert int(efg.argmax(buf[:0]).item()) == 0


def test_lm_head_argmax_single_rank(cuda, oracle):
    """The lm_head shape (Q8_0 32000 x 2048) with the final RMSNorm on one rank: logits
    within 1e-5 of sum|w h| of the reference dot, and the token is their argmax."""
    import torch

    rows, cols = 32000, 2048
    W, x = _make(torch, QType.Q8_0, rows, cols, 21)
    nw = (1 + 0.1 * torch.randn(cols, generator=torch.Generator(device="cuda").manual_seed(4), device="cuda"))
    comm = efg.Comm(efg.Comm.unique_id(), 1, 0)
    try:
        logits = torch.full((rows,), float("nan"), device="cuda")
        tok = torch.full((1,), -1, dtype=torch.int32, device="cuda")
        efg.lm_head_argmax_sharded(QType.Q8_0, logits, tok, W, x, nw, 1e-5, rows, cols, comm)
        torch.cuda.synchronize()
    finally:
        comm.close()
    h = _rmsnorm_host(x.cpu().numpy(), nw.cpu().numpy(), 1e-5)
    _check(oracle, QType.Q8_0, W, torch.from_numpy(h), logits, rows)
    assert int(tok.item()) == oracle.argmax(logits.cpu().numpy())
    assert efg.device_error() == 0


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, cases, out_dir):
    import datetime

    import torch
    import torch.distributed as dist

    torch.cuda.set_device(rank)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    comm = efg.Comm.from_torch()
    try:
        for i, (qt, rows, cols) in enumerate(cases):
            W, x = _make(torch, qt, rows, cols, 11)
            b, c = efg.shard_rows(rows, world, rank)
            shard = W[b:b + c].contiguous()
            # through NCCL (y not registered) ...
            y = torch.full((rows,), float("nan"), device="cuda")
            efg.matvec_sharded(qt, y, shard, x, rows, cols, comm)
            # ... and by the kernel's own peer stores (y registered on every rank), twice in a
            # row, then as a CUDA graph of two calls replayed twice (the epoch lives on the device)
            yf = torch.full((rows + 64,), float("nan"), device="cuda")
            comm.register(yf)
            yv = yf[32:32 + rows]  # the same offset on every rank
            efg.matvec_sharded(qt, yv, shard, x, rows, cols, comm)
            torch.cuda.synchronize()
            first = yv.clone()
            yv.fill_(float("nan"))
            efg.matvec_sharded(qt, yv, shard, x, rows, cols, comm)
            torch.cuda.synchronize()
            second = yv.clone()
            s = torch.cuda.Stream()
            s.wait_stream(torch.cuda.current_stream())
            g = torch.cuda.CUDAGraph()
            with torch.cuda.stream(s), torch.cuda.graph(g, stream=s):
                for _ in range(2):
                    efg.matvec_sharded(qt, yv, shard, x, rows, cols, comm)
            yv.fill_(float("nan"))
            torch.cuda.synchronize()
            g.replay()
            g.replay()
            torch.cuda.synchronize()
            graphed = yv.clone()
            del g
            torch.cuda.synchronize()
            comm.deregister(yf)
            assert torch.isnan(yf[:32]).all() and torch.isnan(yf[32 + rows:]).all()  # nothing outside y
            for tag, t in (("nccl", y), ("fused", first), ("fused2", second), ("graph", graphed)):
                np.save(os.path.join(out_dir, f"y{i}_{tag}_{rank}.npy"), t.cpu().numpy())
            if rank == 0:
                np.save(os.path.join(out_dir, f"W{i}.npy"), W.cpu().numpy())
                np.save(os.path.join(out_dir, f"x{i}.npy"), x.cpu().numpy())
        # lm_head sharded over the ranks with the distributed argmax
        rows, cols = 32000, 2048
        W, x = _make(torch, QType.Q8_0, rows, cols, 23)
        nw = 1 + 0.1 * torch.randn(cols, generator=torch.Generator(device="cuda").manual_seed(4), device="cuda")
        b, c = efg.shard_rows(rows, world, rank)
        shard = W[b:b + c].contiguous()
        logits = torch.empty(c, device="cuda")
        tok = torch.full((1,), -1, dtype=torch.int32, device="cuda")
        efg.lm_head_argmax_sharded(QType.Q8_0, logits, tok, shard, x, nw, 1e-5, rows, cols, comm)
        torch.cuda.synchronize()
        np.save(os.path.join(out_dir, f"lm_logits_{rank}.npy"), logits.cpu().numpy())
        toks = {"nccl": int(tok.item())}
        # the same with a buffer registered: the pairs travel by peer stores inside the argmax
        # launch, twice in a row, as a CUDA graph of two calls replayed twice, and with a NaN in
        # x (every logit NaN: element 0 of the whole vector is NaN, the token is 0)
        reg = torch.zeros(64, device="cuda")
        comm.register(reg)
        for tag in ("peer", "peer2"):
            tok.fill_(-1)
            efg.lm_head_argmax_sharded(QType.Q8_0, logits, tok, shard, x, nw, 1e-5, rows, cols, comm)
            torch.cuda.synchronize()
            toks[tag] = int(tok.item())
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(s), torch.cuda.graph(g, stream=s):
            for _ in range(2):
                efg.lm_head_argmax_sharded(QType.Q8_0, logits, tok, shard, x, nw, 1e-5, rows, cols, comm)
        tok.fill_(-1)
        torch.cuda.synchronize()
        g.replay()
        g.replay()
        torch.cuda.synchronize()
        toks["graph"] = int(tok.item())
        del g
        x_nan = x.clone()
        x_nan[5] = float("nan")
        efg.lm_head_argmax_sharded(QType.Q8_0, logits, tok, shard, x_nan, nw, 1e-5, rows, cols, comm)
        torch.cuda.synchronize()
        toks["nan"] = int(tok.item())
        comm.deregister(reg)
        np.save(os.path.join(out_dir, f"lm_tok_{rank}.npy"), np.array([toks[k] for k in ("nccl", "peer", "peer2", "graph", "nan")]))
        assert efg.device_error() == 0
    finally:
        comm.close()
        dist.barrier()
        dist.destroy_process_group()


def test_multi_rank(tmp_path, oracle):
    import torch
    import torch.multiprocessing as mp

    n = min(torch.cuda.device_count(), 8)
    if n < 2:
        pytest.skip("needs two GPUs")
    # shards on the tensor-core kernel (>= 48 MB each at 2 ranks), the CUDA-core kernel, a
    # ragged split, and the generic kernel (cols % 64 != 0)
    cases = [(QType.Q4_0, 24576, 8192), (QType.Q4_0, 16384, 8192), (QType.Q4_0, 1001, 256),
             (QType.Q8_0, 4099, 2048), (QType.Q8_0, 515, 96)]
    mp.start_processes(_rank_main, args=(n, _free_port(), cases, str(tmp_path)), nprocs=n, join=True,
                       start_method="spawn")
    from conftest import rel_dot_errors

    for i, (qt, rows, cols) in enumerate(cases):
        ys = [np.load(tmp_path / f"y{i}_{tag}_{r}.npy") for tag in ("nccl", "fused", "fused2", "graph")
              for r in range(n)]
        for y in ys[1:]:  # every path, every rank, every call: the same bits
            np.testing.assert_array_equal(y, ys[0])
        W, x = np.load(tmp_path / f"W{i}.npy"), np.load(tmp_path / f"x{i}.npy")
        err = rel_dot_errors(oracle, qt, W, x, rows, ys[0])
        assert err.max() <= TOL, (i, err.max())
    # the distributed argmax, through NCCL and through the peer exchange (twice, in a graph):
    # the same token on every rank, the argmax of all shards' logits; 0 when x holds a NaN
    full = np.concatenate([np.load(tmp_path / f"lm_logits_{r}.npy") for r in range(n)])
    want = oracle.argmax(full)
    for r in range(n):
        toks = np.load(tmp_path / f"lm_tok_{r}.npy")
        assert list(toks[:4]) == [want] * 4 and toks[4] == 0, (r, toks, want)
