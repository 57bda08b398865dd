"""N-split host logic on CPU ranks (gloo, world size 2): the column partition of
clove_nsplit_col_begin, per-rank shard GEMMs (oracle on CPU), the all-gather and
the column re-layout that clove_nsplit_gemm_* perform on GPUs -- plus a rank that
fails before the collective, which the other rank must see as an error within its
process-group timeout instead of hanging."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _relayout(slots, N, P, Nmax):
    """Same scatter as relayout_columns_kernel: slot p -> columns of rank p."""
    import clove_compute_b200 as cc
    M = slots.shape[1]
    C = np.empty((M, N), slots.dtype)
    for p in range(P):
        c0, c1 = cc.col_begin(N, P, p), cc.col_begin(N, P, p + 1)
        C[:, c0:c1] = slots[p, :, : c1 - c0]
    return C


def _worker(rank, world, port, M, N, K, fail_rank, q):
    import sys
    sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=5))
    try:
        import clove_compute_b200 as cc
        import oracle
        from clove_compute_b200 import workloads as wl
        A, B = wl.fp16_operands(M, N, K, seed=3)
        c0, c1 = cc.col_begin(N, world, rank), cc.col_begin(N, world, rank + 1)
        shard = oracle.gemm_fp16(A, np.ascontiguousarray(B[:, c0:c1]))
        if rank == fail_rank:
            raise RuntimeError("injected failure before the all-gather")
        Nmax = (N + world - 1) // world
        pad = np.zeros((M, Nmax), np.float16)
        pad[:, : c1 - c0] = shard
        out = [torch.empty((M, Nmax), dtype=torch.float16) for _ in range(world)]
        dist.all_gather(out, torch.from_numpy(pad))
        C = _relayout(np.stack([o.numpy() for o in out]), N, world, Nmax)
        ref = oracle.gemm_fp16(A, B)
        q.put((rank, "ok", bool(np.array_equal(C.view(np.uint16), ref.view(np.uint16)))))
    except Exception as e:  # report, never hang
        q.put((rank, "error", type(e).__name__ + ": " + str(e)[:200]))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _run(M, N, K, fail_rank=-1, world=2):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, M, N, K, fail_rank, q))
             for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        r, kind, val = q.get(timeout=120)
        res[r] = (kind, val)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return res


@pytest.mark.parametrize("M,N,K", [(64, 96, 64), (32, 7, 48)])
def test_nsplit_gather_relayout_matches_full_gemm(oracle_mod, clove_lib, M, N, K):
    res = _run(M, N, K)
    assert res == {0: ("ok", True), 1: ("ok", True)}


def test_nsplit_rank_failure_is_reported_not_hung(oracle_mod, clove_lib):
    res = _run(32, 64, 32, fail_rank=1)
    assert res[1][0] == "error" and "injected" in res[1][1]
    assert res[0][0] == "error"  # the survivor's collective ends with an error
