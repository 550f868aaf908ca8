"""The decode path as a CUDA graph: one eager call, capture of moe_solve_v2,
then replays on new tokens copied into the layer's x must give bit-identical
results to eager calls on the same tokens (16-bit and 4-bit formats, a
many-expert sliced router included), and each replay's routing and output
must match the CPU oracle on those tokens (bit-exact routing, the format's
max-abs-rel bar)."""
import numpy as np
import pytest
import torch

import sparsemoe_b200 as sm
from oracle import oracle as O

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("cfg", [
    sm.LayerConfig(1, 64, 512, 256, 8, 2, 1.25, dtype=sm.DTYPE_BF16),
    sm.LayerConfig(1, 128, 1024, 512, 32, 8, 1.25, dtype=sm.DTYPE_W4A16, router_f32=True, zipf_s=1.0),
    sm.LayerConfig(1, 96, 512, 256, 64, 6, 1.0, dtype=sm.DTYPE_NVFP4, router_f32=True, zipf_s=1.1),
], ids=["bf16", "int4_g128", "nvfp4_e64"])
def test_graph_replay_matches_eager(gpu, cfg):
    inp = sm.make_inputs(cfg, 0)
    eager = sm.MoeLayer(cfg, gpu).load(inp)
    graphed = sm.MoeLayer(cfg, gpu).load(inp)
    graphed.capture()
    for seed in (1, 2, 3):
        x = sm.make_inputs(cfg, seed)["x"]
        xt = torch.from_numpy(x.view(np.int16)).view(eager.x.dtype).to(gpu)
        eager.x[: cfg.T].copy_(xt)
        graphed.x[: cfg.T].copy_(xt)
        eager.forward()
        graphed.replay()
        torch.cuda.synchronize()
        eager.sync_check()
        assert torch.equal(eager.idx, graphed.idx)
        assert torch.equal(eager.out, graphed.out), f"seed {seed}: graph replay differs from eager"
        ref = O.forward({**inp, "x": x}, cfg)
        assert np.array_equal(graphed.idx.cpu().numpy()[: cfg.T], ref["idx"])
        out = graphed.out.cpu().numpy()[: cfg.T]
        tol = 6e-2 if cfg.w4 else 1e-2
        assert float(np.abs(out - ref["out"]).max() / np.abs(ref["out"]).max()) <= tol
