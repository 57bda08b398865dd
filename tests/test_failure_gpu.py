"""Failure detection without a GPU fault: every cross-GPU wait in this library is
bounded. A two-rank completion wait whose other rank never signals must run out
after its limit, record device error 1 (a bounded wait expired) and return, leaving
the context usable for the next call."""
import time

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_cross_rank_wait_runs_out_and_reports(clove_lib, cuda, oracle_mod):
    cc = clove_lib
    assert cc.device_error() == 0
    words = torch.full((8,), -1, dtype=torch.int64, device="cuda")
    t0 = time.perf_counter()
    cc.debug_peer_wait_timeout(words, 20_000_000)  # 20 ms limit
    err = cc.device_error()  # synchronises
    dt = time.perf_counter() - t0
    assert err == 1, err
    assert 0.015 < dt < 1.9, dt  # ran out at its own limit, not the product's 2 s
    w = words.cpu().tolist()
    # epoch 1; this rank published into its own slot and the absent rank's array;
    # the slot it waited on stayed 0.
    assert w[0] == 1 and w[1] == 1 and w[3] == 1 and w[2] == 0, w
    assert cc.device_error() == 0  # read-and-clear

    # The context stays usable: a GEMM afterwards is correct and error-free.
    from clove_compute_b200 import workloads as wl
    A, B = wl.fp16_operands(256, 256, 512, seed=4)
    C = cc.gemm_fp16(torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda())
    ref = oracle_mod.gemm_fp16(A, B)
    e = np.linalg.norm(C.cpu().numpy().astype(np.float64) - ref) / np.linalg.norm(ref)
    assert e < 1e-2
    assert cc.device_error() == 0


def test_peer_wait_hook_rejects_bad_arguments(clove_lib, cuda):
    cc = clove_lib
    words = torch.zeros(8, dtype=torch.int64, device="cuda")
    with pytest.raises(cc.CloveError):
        cc.debug_peer_wait_timeout(words, 0)
    with pytest.raises(cc.CloveError):
        cc.debug_peer_wait_timeout(words, 3_000_000_000)  # above the product bound
