"""Failure detection on the GPU without a GPU fault.

* A bounded device wait is made to run out (an mbarrier nothing arrives on):
  the kernel records a timeout in the status word and returns; the host reads
  MOE_ERR_TIMEOUT, and the context stays usable for the next layer call.
* (>= 2 GPUs) an expert-parallel rank leaves between steps, with none of its
  kernels or collectives in flight; the survivor's next forward() raises
  PeerLost on the host (PeerWatch) before it enqueues anything.  NCCL
  transport, NVLS off, no peer mappings."""
import ctypes
import os
import time

import numpy as np
import pytest

import sparsemoe_b200 as sm
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def test_bounded_wait_times_out_and_context_survives(gpu):
    import torch
    s = torch.cuda.current_stream()
    t0 = time.time()
    sm.check(sm.lib.moe_selftest_wait_timeout(50_000_000, ctypes.c_void_p(s.cuda_stream)))   # 50 ms
    rc = sm.lib.moe_check_device_status(ctypes.c_void_p(s.cuda_stream))
    assert rc == sm.MOE_ERR_TIMEOUT
    assert "timed out" in sm.last_error()
    assert time.time() - t0 < 10
    # the context is intact: a layer call runs, clears the status word and matches the oracle
    cfg = sm.LayerConfig(1, 128, 256, 256, 8, 2, 1.25)
    inp = sm.make_inputs(cfg, 0)
    L = sm.MoeLayer(cfg, gpu).load(inp)
    L.forward()
    L.sync_check()
    ref = O.forward(inp, cfg)
    assert np.array_equal(L.idx.cpu().numpy(), ref["idx"])


def _leave_worker(rank, world, port, results):
    import datetime
    import torch
    import torch.distributed as dist
    from sparsemoe_b200.ep import ExpertParallelLayer
    from sparsemoe_b200.health import PeerLost
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30),
                            device_id=torch.device("cuda", rank))
    cfg = sm.LayerConfig(1, 128, 256, 256, 8, 2, 1.25, dtype=sm.DTYPE_BF16)
    full = sm.make_inputs(cfg, 5)
    ep = ExpertParallelLayer(cfg, f"cuda:{rank}", transport="nccl", health_timeout=3.0).load(
        {**full, "x": sm.make_inputs(cfg, 100 + rank)["x"]})
    ep.forward()
    ep.sync_check()                                  # step 0 done everywhere, nothing in flight
    if rank == world - 1:
        results[rank] = "left"
        os._exit(0)                                  # leaves between steps
    t0 = time.time()
    try:
        ep.forward()
        results[rank] = ("completed", time.time() - t0)
    except PeerLost as e:
        torch.cuda.synchronize()
        results[rank] = ("peer_lost", time.time() - t0, e.missing)
    os._exit(0)


def test_ep_rank_leaving_between_steps(gpu):
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("needs >= 2 GPUs")
    port = 29700 + os.getpid() % 200
    with mp.Manager() as m:
        res = m.dict()
        ctx = mp.spawn(_leave_worker, args=(2, port, res), nprocs=2, join=False)
        t_end = time.time() + 120
        while not ctx.join(timeout=5):
            assert time.time() < t_end, "ranks still running"
        res = dict(res)
    assert res[1] == "left"
    status, dt, missing = res[0]
    assert status == "peer_lost" and missing == [1] and dt < 20, res[0]
