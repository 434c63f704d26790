"""Multi-rank host logic on CPU with gloo (world size 2): row sharding, the
max-over-ranks timing reduction and host-side failure detection."""
import os
import socket
import sys
import traceback

import numpy as np
import pytest
import torch.multiprocessing as mp

from conftest import PKG_PARENT, ROOT


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port):
    for p in (ROOT, PKG_PARENT):
        if p not in sys.path:
            sys.path.insert(0, p)
    import datetime
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=20))
    return dist


def _sharded_dense_worker(rank, world, port, errq):
    try:
        dist = _init(rank, world, port)
        import torch
        import oracle
        from mlir_edsl.sharding import max_over_ranks, row_shards
        M, N, K = 203, 70, 90  # not divisible by the world size
        rng = np.random.default_rng(0)
        X = rng.uniform(-1, 1, (M, K)).astype(np.float32)
        W = rng.uniform(-1, 1, (K, N)).astype(np.float32)
        b = rng.uniform(-1, 1, (N,)).astype(np.float32)
        r0, rows = row_shards(M, world)[rank]
        Yloc = oracle.dense_f32(X[r0:r0 + rows], W, b, act=oracle.ACT_RELU)
        sizes = [s[1] for s in row_shards(M, world)]
        pad = max(sizes)  # equal-size all_gather of padded shards, trimmed after
        buf = torch.zeros((pad, N))
        buf[:rows] = torch.from_numpy(Yloc)
        gathered = [torch.empty((pad, N)) for _ in sizes]
        dist.all_gather(gathered, buf)
        Y = torch.cat([g[:s] for g, s in zip(gathered, sizes)]).numpy()
        full = oracle.dense_f32(X, W, b, act=oracle.ACT_RELU)
        np.testing.assert_array_equal(Y, full)  # row shards are bit-identical
        t = max_over_ranks(1.0 + rank, dist)
        assert t == float(world), t
        dist.destroy_process_group()
    except Exception:
        errq.put((rank, traceback.format_exc()))


def _gather_pipelined_worker(rank, world, port, errq):
    """Slab-pipelined all-gather of a row-sharded dense layer (the host logic
    of dense_rows(..., gather=True)); the compute callback is the oracle."""
    try:
        dist = _init(rank, world, port)
        import torch
        import oracle
        from mlir_edsl.sharding import gather_rows_pipelined
        rows, N, K = 37, 20, 16  # rows per rank; 37 rows in 4 uneven slabs
        rng = np.random.default_rng(5)
        X = rng.uniform(-1, 1, (world * rows, K)).astype(np.float32)
        W = rng.uniform(-1, 1, (K, N)).astype(np.float32)
        calls = []

        def compute(r0, r1, out):
            calls.append((r0, r1))
            xs = X[rank * rows + r0: rank * rows + r1]
            out.copy_(torch.from_numpy(oracle.dense_f32(xs, W, act=oracle.ACT_RELU)))

        Y = gather_rows_pipelined(rows, N, compute, slabs=4, dtype=torch.float32)
        assert calls == [(0, 10), (10, 19), (19, 28), (28, 37)], calls
        np.testing.assert_array_equal(Y.numpy(), oracle.dense_f32(X, W, act=oracle.ACT_RELU))
        dist.destroy_process_group()
    except Exception:
        errq.put((rank, traceback.format_exc()))


def _failing_rank_worker(rank, world, port, errq):
    """Rank 1 fails before the barrier; rank 0 must learn it through a bounded
    monitored barrier instead of hanging."""
    try:
        dist = _init(rank, world, port)
        import datetime
        if rank == 1:
            raise SystemExit(3)  # leaves between steps, nothing in flight
        try:
            dist.monitored_barrier(timeout=datetime.timedelta(seconds=3))
            errq.put((rank, "barrier unexpectedly succeeded"))
        except RuntimeError as e:
            if "1" not in str(e):
                errq.put((rank, f"failure message does not name rank 1: {e}"))
    except SystemExit:
        pass
    except Exception:
        errq.put((rank, traceback.format_exc()))


def _unequal_rows_worker(rank, world, port, errq):
    """Gathered dense layer with 3 rows on rank 0 and 2 on rank 1: every rank
    raises the same ValueError before any buffer exchange or native call."""
    try:
        _init(rank, world, port)
        import torch
        import torch.distributed as dist
        from mlir_edsl.sharding import dense_rows
        rows = 3 - rank
        X = torch.zeros((rows, 8))
        W = torch.zeros((8, 4))
        for transport in ("fused", "ce", "nccl"):
            try:
                dense_rows(X, W, None, 1, 0.0, gather=True, transport=transport)
                errq.put((rank, f"{transport}: unequal rows accepted"))
            except ValueError as e:
                if "same rows" not in str(e) or "2..3" not in str(e):
                    errq.put((rank, f"{transport}: unexpected message {e}"))
        dist.barrier()  # both ranks are still in step
        dist.destroy_process_group()
    except Exception:
        errq.put((rank, traceback.format_exc()))


def _spawn(fn, world=2):
    ctx = mp.get_context("spawn")
    errq = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=fn, args=(r, world, port, errq)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    for p in procs:
        if p.is_alive():
            p.kill()
            pytest.fail("worker did not finish")
    errs = []
    while not errq.empty():
        errs.append(errq.get())
    return errs


def test_row_shards_partition():
    from mlir_edsl.sharding import row_shards
    for M in (0, 1, 7, 65536, 65537):
        for n in (1, 2, 3, 8):
            sh = row_shards(M, n)
            assert sum(r for _, r in sh) == M
            assert all(sh[i][0] + sh[i][1] == sh[i + 1][0] for i in range(n - 1))
            assert max(r for _, r in sh) - min(r for _, r in sh) <= 1


def test_sharded_dense_gloo_world2():
    errs = _spawn(_sharded_dense_worker)
    assert not errs, errs


def test_failed_rank_is_detected_gloo_world2():
    errs = _spawn(_failing_rank_worker)
    assert not errs, errs


def test_slab_pipelined_gather_gloo_world2():
    errs = _spawn(_gather_pipelined_worker)
    assert not errs, errs


def test_slab_bounds():
    from mlir_edsl.sharding import slab_bounds
    for rows in (1, 5, 37, 8192):
        for slabs in (1, 3, 4, 100):
            b = slab_bounds(rows, slabs)
            assert b[0][0] == 0 and b[-1][1] == rows
            assert all(b[i][1] == b[i + 1][0] for i in range(len(b) - 1))
            assert all(r1 > r0 for r0, r1 in b)
            sizes = [r1 - r0 for r0, r1 in b]
            assert max(sizes) - min(sizes) <= 1


def test_fused_output_bases():
    """Each rank's rows land at row rank * rows of every buffer: its own and,
    for the fused transport's epilogue stores, each peer's (never its own
    twice), so the world's regions tile every buffer exactly once."""
    for p in (ROOT, PKG_PARENT):
        if p not in sys.path:
            sys.path.insert(0, p)
    from mlir_edsl.sharding import fused_output_bases
    rows, N = 1000, 768
    for world in (2, 3, 8):
        size = world * rows * N * 4
        ptrs = [0x7f0000000000 + r * (1 << 36) for r in range(world)]
        written = {r: [] for r in range(world)}  # buffer -> regions stored into it
        for rank in range(world):
            own, peers = fused_output_bases(ptrs, rank, rows, N)
            assert len(peers) == world - 1 <= 7
            for base in [own] + peers:
                owner = max(r for r in range(world) if ptrs[r] <= base)
                assert base + rows * N * 4 <= ptrs[owner] + size
                written[owner].append(base - ptrs[owner])
            assert own == ptrs[rank] + rank * rows * N * 4
        for r in range(world):
            assert sorted(written[r]) == [q * rows * N * 4 for q in range(world)]



def test_gathered_unequal_rows_rejected_on_every_rank_gloo_world2():
    errs = _spawn(_unequal_rows_worker)
    assert not errs, errs
