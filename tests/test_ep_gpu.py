"""Expert parallelism on real GPUs (NCCL): each rank routes its own tokens,
sends rows (and, for the dynamically quantised formats, their row scales) to
the experts' owners, runs its E/P experts, gets the rows back and combines.
Must equal the single-GPU layer on the same tokens bit for bit, and match the
CPU oracle (routing bit-exact, the format's bar).  Needs >= 2 GPUs; runs as
child processes, one per GPU, with NVLS off."""
import os

import numpy as np
import pytest

import sparsemoe_b200 as sm

pytestmark = pytest.mark.gpu


def _worker(rank, world, port, case, results):
    import torch
    import torch.distributed as dist
    from sparsemoe_b200.ep import ExpertParallelLayer
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    from datetime import timedelta
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    B, N, d, f, E, k, cf, dtype, zipf, chunks, glob = case[:11]
    transport = case[11] if len(case) > 11 else "nccl"
    placement = case[12] if len(case) > 12 else "contiguous"
    if glob:
        # one batch of world*N tokens; this rank holds tokens [rank*N, (rank+1)*N) of every batch
        full_cfg = sm.LayerConfig(B, N * world, d, f, E, k, cf, dtype=dtype, zipf_s=zipf,
                                  router_f32=dtype in (sm.DTYPE_W4A16, sm.DTYPE_NVFP4))
        full = sm.make_inputs(full_cfg, 5)
        x = full["x"].reshape(B, world, N, d)[:, rank].reshape(B * N, d)
        cfg = sm.LayerConfig(B, N, d, f, E, k, cf, dtype=dtype, zipf_s=zipf, router_f32=full_cfg.router_f32)
        ep = ExpertParallelLayer(cfg, f"cuda:{rank}", global_batch=True, transport=transport,
                                 placement=placement).load({**full, "x": x})
        single = sm.MoeLayer(full_cfg, f"cuda:{rank}").load(full)
        single_inputs = full
        rows = np.concatenate([np.arange(b * N * world + rank * N, b * N * world + (rank + 1) * N)
                               for b in range(B)])
    else:
        cfg = sm.LayerConfig(B, N, d, f, E, k, cf, dtype=dtype, zipf_s=zipf)
        full = sm.make_inputs(cfg, 5)
        mine = sm.make_inputs(cfg, 100 + rank)
        inputs = {**full, "x": mine["x"]}
        ep = ExpertParallelLayer(cfg, f"cuda:{rank}", chunks=chunks, transport=transport,
                                 placement=placement).load(inputs)
        single = sm.MoeLayer(cfg, f"cuda:{rank}").load(inputs)
        single_inputs = inputs
        rows = np.arange(cfg.T)
    ep.forward()
    ep.sync_check()
    ep.forward()          # second call: reuses buffers and the library scratch
    ep.sync_check()
    single.forward()
    single.sync_check()
    a = ep.out.cpu().numpy()[: cfg.T]
    b = single.out.cpu().numpy()[rows]
    idx_equal = bool(np.array_equal(ep.idx.cpu().numpy()[: cfg.T], single.idx.cpu().numpy()[rows]))
    # and against the CPU oracle on the same tokens (this rank's rows of the single-GPU problem)
    from oracle import oracle as O
    sc = single.cfg
    ref = O.forward(single_inputs, sc)
    oracle_idx = bool(np.array_equal(ep.idx.cpu().numpy()[: cfg.T], ref["idx"][rows]))
    tol = {sm.DTYPE_F16: 1e-2, sm.DTYPE_BF16: 1e-2, sm.DTYPE_W4A16: 6e-2, sm.DTYPE_NVFP4: 6e-2}.get(dtype, 3e-2)
    oracle_err = float(np.abs(a - ref["out"][rows]).max() / max(np.abs(ref["out"][rows]).max(), 1e-30))
    results[rank] = (bool(np.array_equal(a, b)), float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30)),
                     idx_equal, oracle_idx and oracle_err <= tol)
    ep.close()
    dist.destroy_process_group()


CASES = {
    "bf16": (2, 256, 512, 512, 8, 2, 1.25, sm.DTYPE_BF16, 0.0, 1, False),
    "fp16_zipf_drops": (1, 384, 256, 256, 16, 4, 1.0, sm.DTYPE_F16, 1.1, 1, False),
    "int8": (2, 128, 512, 256, 8, 2, 1.25, sm.DTYPE_INT8, 0.0, 1, False),
    "two_chunks": (4, 128, 256, 256, 8, 2, 1.25, sm.DTYPE_BF16, 0.0, 2, False),
    "int8_channel": (1, 256, 512, 256, 16, 4, 1.0, sm.DTYPE_INT8_CHANNEL, 1.1, 1, False),
    "fp8_block": (1, 256, 512, 256, 16, 4, 1.25, sm.DTYPE_FP8_BLOCK, 0.0, 1, False),
    "int4_g128": (1, 256, 512, 256, 16, 4, 1.25, sm.DTYPE_W4A16, 1.0, 1, False),
    "nvfp4": (1, 256, 512, 256, 16, 4, 1.25, sm.DTYPE_NVFP4, 1.0, 1, False),
    "global_bf16_drops": (2, 192, 512, 256, 16, 4, 1.0, sm.DTYPE_BF16, 1.2, 1, True),
    "global_int4_deepseek_like": (1, 256, 512, 256, 32, 8, 1.25, sm.DTYPE_W4A16, 1.0, 1, True),
    "global_fp8": (1, 256, 512, 256, 16, 4, 1.0, sm.DTYPE_FP8_BLOCK, 1.1, 1, True),
    # rows over NVLink peer memory: copy-engine dispatch, down-GEMM epilogue stores into the senders
    "peer_bf16": (2, 256, 512, 512, 8, 2, 1.25, sm.DTYPE_BF16, 0.0, 1, False, "peer"),
    "peer_fp8_block_scales": (1, 256, 512, 256, 16, 4, 1.25, sm.DTYPE_FP8_BLOCK, 0.0, 1, False, "peer"),
    "peer_global_int4": (1, 256, 512, 256, 32, 8, 1.25, sm.DTYPE_W4A16, 1.0, 1, True, "peer"),
    "peer_global_nvfp4_drops": (1, 192, 512, 256, 16, 4, 1.0, sm.DTYPE_NVFP4, 1.2, 1, True, "peer"),
    # strided expert ownership (rank q holds experts q, q+P, ...)
    "peer_strided_bf16": (2, 256, 512, 512, 8, 2, 1.25, sm.DTYPE_BF16, 0.0, 1, False, "peer", "strided"),
    "peer_strided_global_int8ch_zipf": (1, 256, 512, 256, 32, 8, 1.0, sm.DTYPE_INT8_CHANNEL, 1.0, 1, True, "peer",
                                        "strided"),
}


@pytest.mark.parametrize("name", list(CASES))
def test_ep_matches_single_gpu(gpu, name):
    import torch
    import torch.multiprocessing as mp
    case = CASES[name]
    world = torch.cuda.device_count()
    if world < 2:
        pytest.skip("needs >= 2 GPUs")
    world = 2 if case[4] % 4 else min(world, 4)
    port = 29600 + (os.getpid() % 2000)
    with mp.Manager() as m:
        results = m.dict()
        mp.spawn(_worker, args=(world, port, case, results), nprocs=world, join=True)
        res = dict(results)
    assert len(res) == world
    for rank, (equal, err, idx_equal, oracle_ok) in res.items():
        assert idx_equal, f"rank {rank}: routing differs"
        assert err < 1e-6, f"rank {rank}: max-abs-rel {err}"
        assert oracle_ok, f"rank {rank}: differs from the CPU oracle"



@pytest.mark.parametrize("strided", [False, True])
def test_ep_plan_kernel_matches_host(gpu, strided):
    """moe_ep_plan (one-CTA kernel) against its host restatement on random
    kept-row tables, every rank of an 8-way layout (runs on one GPU)."""
    import ctypes
    import torch
    from sparsemoe_b200.ep import ep_plan_host
    rng = np.random.default_rng(1)
    P, E = 8, 64
    table = rng.integers(0, 300, (P, E)).astype(np.int32)
    t = torch.from_numpy(table).to(gpu)
    plan = torch.empty(7 * E, dtype=torch.int32, device=gpu)
    for rank in range(P):
        rc = sm.lib.moe_ep_plan(ctypes.c_void_p(t.data_ptr()), P, rank, E, int(strided),
                                ctypes.c_void_p(plan.data_ptr()), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
        assert rc == 0
        torch.cuda.synchronize()
        assert np.array_equal(plan.cpu().numpy(), ep_plan_host(table, rank, strided)), f"rank {rank}"
