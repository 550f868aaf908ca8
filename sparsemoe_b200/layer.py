"""MoeLayer: device buffers for one layer shape plus the call into the C ABI.

PyTorch allocates the device memory (the reference's allocator role,
inputs/data.cu:199-524); every computation runs in libsparsemoe_b200.so.
"""
from __future__ import annotations

import ctypes

import numpy as np
import torch

from . import LayerConfig, MoEArgs, check, lib


def _t16(cfg: LayerConfig):
    return torch.bfloat16 if cfg.act_bf16 else torch.float16


class MoeLayer:
    def __init__(self, cfg: LayerConfig, device: str | torch.device = "cuda", want_logits: bool = True,
                 want_out16: bool = True):
        self.cfg = cfg
        self.device = torch.device(device)
        B, N, d, f, E, k = cfg.num_batches, cfg.tokens, cfg.d_model, cfg.d_ff, cfg.num_experts, cfg.top_k
        cap = cfg.capacity()
        self.cap = cap
        t16 = _t16(cfg)
        dev = self.device
        rows = max(B * E * cap, 1)
        T = cfg.T
        z = lambda *s, dt: torch.empty(*s, dtype=dt, device=dev)  # noqa: E731
        self.x = z(max(T, 1), d, dt=t16)
        self.wr = z(d, E, dt=torch.float32 if cfg.router_f32 else t16)
        wt = torch.int8 if (cfg.int8 or cfg.int8ch or cfg.int4ptx) else \
            (torch.uint8 if (cfg.fp8 or cfg.fp8pt) else t16)
        if cfg.int4ptx:
            # the reference's packed-transposed int4: per expert [N/2][K] bytes
            self.wg = z(E, f // 2, d, dt=torch.uint8)
            self.wu = z(E, f // 2, d, dt=torch.uint8)
            self.wd = z(E, d // 2, f, dt=torch.uint8)
        elif cfg.w4:
            self.wg = z(E, d, f // 2, dt=torch.uint8)
            self.wu = z(E, d, f // 2, dt=torch.uint8)
            self.wd = z(E, f, d // 2, dt=torch.uint8)
        else:
            self.wg = z(E, d, f, dt=wt)
            self.wu = z(E, d, f, dt=wt)
            self.wd = z(E, f, d, dt=wt)
        self.scales = {}
        self.bias = None
        self.logits = z(max(T, 1), E, dt=torch.float32) if want_logits else None
        self.idx = z(max(T, 1), k, dt=torch.int32)
        self.w = z(max(T, 1), k, dt=torch.float32)
        self.counts = z(max(B, 1), E, dt=torch.int32)
        self.token_ids = z(rows, dt=torch.int32)
        self.token_weights = z(rows, dt=torch.float32)
        self.a_rows = z(rows, d, dt=wt)
        self.h_rows = z(rows, f, dt=wt)
        self.y_rows = z(rows, d, dt=torch.float32)
        self.out = z(max(T, 1), d, dt=torch.float32)
        self.out16 = z(max(T, 1), d, dt=t16) if want_out16 else None
        # the stages either side (MoeDims.norm_* / residual): set by load() when the inputs carry them
        self.norm_w = self.xn = self.residual = None
        self.norm_eps = 0.0

    # -- inputs ---------------------------------------------------------------
    def load(self, inputs: dict) -> "MoeLayer":
        """Copies host inputs from make_inputs() (uint16 bit patterns) to the device."""
        def put(dst: torch.Tensor, arr: np.ndarray):
            arr = np.ascontiguousarray(arr)
            if arr.dtype == np.uint16:
                src = torch.from_numpy(arr.view(np.int16)).view(dst.dtype)
            else:
                src = torch.from_numpy(arr)
            dst.copy_(src.reshape(dst.shape), non_blocking=False)
        if self.cfg.T > 0:
            put(self.x, inputs["x"])
        put(self.wr, inputs["wr"])
        sfx = "_q" if (self.cfg.per_tensor or self.cfg.int8ch or self.cfg.fp8 or self.cfg.w4) else ""
        put(self.wg, inputs["wg" + sfx])
        put(self.wu, inputs["wu" + sfx])
        put(self.wd, inputs["wd" + sfx])
        if self.cfg.per_tensor:
            self.scales = {k: inputs[k] for k in ("s_in", "s_gate", "s_up", "s_mid", "s_down")}
        if self.cfg.nvfp4:
            self.w4sz = [torch.from_numpy(np.ascontiguousarray(inputs[k])).to(self.device)
                         for k in ("wg_s", "wu_s", "wd_s")]
            self.fp4g = [torch.from_numpy(np.ascontiguousarray(inputs[k], np.float32)).to(self.device)
                         for k in ("wg_g", "wu_g", "wd_g")]
        elif self.cfg.w4:
            self.w4sz = [torch.from_numpy(np.ascontiguousarray(inputs[k]).view(np.int16)).to(self.device)
                         for k in ("wg_s", "wu_s", "wd_s", "wg_z", "wu_z", "wd_z")]
        if self.cfg.channel_scaled:
            self.wscale = [torch.from_numpy(np.ascontiguousarray(inputs[k])).to(self.device)
                           for k in ("sg", "su", "sd")]
        if inputs.get("bias") is not None:
            self.bias = torch.from_numpy(inputs["bias"]).to(self.device)
        if inputs.get("norm_w") is not None:       # pre-MoE RMSNorm of x (gamma [d], 16-bit)
            self.norm_w = torch.empty(self.cfg.d_model, dtype=self.x.dtype, device=self.device)
            put(self.norm_w, inputs["norm_w"])
            self.norm_eps = float(inputs.get("norm_eps", 1e-6))
            self.xn = torch.empty_like(self.x)
        if inputs.get("residual") is not None:     # added to every output row in the combine
            self.residual = torch.empty_like(self.x)
            if self.cfg.T > 0:
                put(self.residual, inputs["residual"])
        return self

    # -- call -----------------------------------------------------------------
    def args(self) -> MoEArgs:
        a = MoEArgs()
        p = lambda t: None if t is None else t.data_ptr()  # noqa: E731
        a.input = p(self.x)
        a.router_weights = p(self.wr)
        if self.cfg.w4:
            a.expert_up_proj_weights_int4 = p(self.wu)
            a.expert_gate_proj_weights_int4 = p(self.wg)
            a.expert_down_proj_weights_int4 = p(self.wd)
            a.per_expert_wmma_inputs = p(self.a_rows)
            a.hidden_mlp_layer_1_out_fp16 = p(self.h_rows)
        elif self.cfg.fp8:
            a.expert_up_proj_weights_fp8 = p(self.wu)
            a.expert_gate_proj_weights_fp8 = p(self.wg)
            a.expert_down_proj_weights_fp8 = p(self.wd)
            a.per_expert_wmma_inputs_fp8 = p(self.a_rows)
            a.hidden_mlp_layer_1_out_fp8 = p(self.h_rows)
        elif self.cfg.int8ch:
            a.expert_up_proj_weights_int8 = p(self.wu)
            a.expert_gate_proj_weights_int8 = p(self.wg)
            a.expert_down_proj_weights_int8 = p(self.wd)
            a.per_expert_wmma_inputs_int8 = p(self.a_rows)
            a.hidden_mlp_layer_1_out_int8 = p(self.h_rows)
        elif self.cfg.per_tensor:
            if self.cfg.int4ptx:
                a.expert_up_proj_weights_int4 = p(self.wu)
                a.expert_gate_proj_weights_int4 = p(self.wg)
                a.expert_down_proj_weights_int4 = p(self.wd)
            elif self.cfg.fp8pt:
                a.expert_up_proj_weights_fp8 = p(self.wu)
                a.expert_gate_proj_weights_fp8 = p(self.wg)
                a.expert_down_proj_weights_fp8 = p(self.wd)
            else:
                a.expert_up_proj_weights_int8 = p(self.wu)
                a.expert_gate_proj_weights_int8 = p(self.wg)
                a.expert_down_proj_weights_int8 = p(self.wd)
            if self.cfg.fp8pt:
                a.per_expert_wmma_inputs_fp8 = p(self.a_rows)
                a.hidden_mlp_layer_1_out_fp8 = p(self.h_rows)
            else:
                a.per_expert_wmma_inputs_int8 = p(self.a_rows)
                a.hidden_mlp_layer_1_out_int8 = p(self.h_rows)
            sc = self.scales
            a.scale_input_act, a.scale_gate_w, a.scale_up_w = sc["s_in"], sc["s_gate"], sc["s_up"]
            a.scale_mid_act, a.scale_down_w = sc["s_mid"], sc["s_down"]
        else:
            a.expert_up_proj_weights = p(self.wu)
            a.expert_gate_proj_weights = p(self.wg)
            a.expert_down_proj_weights = p(self.wd)
            a.per_expert_wmma_inputs = p(self.a_rows)
            a.hidden_mlp_layer_1_out_fp16 = p(self.h_rows)
        a.expert_logits = p(self.logits)
        a.selected_expert_indices = p(self.idx)
        a.selected_expert_weights = p(self.w)
        a.expert_counts = p(self.counts)
        a.expert_token_ids = p(self.token_ids)
        a.expert_token_weights = p(self.token_weights)
        a.hidden_mlp_layer_2_out = p(self.y_rows)
        a.final_output = p(self.out)
        a.num_batches = self.cfg.num_batches
        a.use_capacity = self.cfg.cap >= 0
        a.cap = self.cap
        return a

    def dims(self):
        ws = tuple(t.data_ptr() for t in self.wscale) if self.cfg.channel_scaled else (None, None, None)
        w4 = tuple(t.data_ptr() for t in self.w4sz) if self.cfg.w4 else ()
        w4 = w4 + (None,) * (6 - len(w4))
        g4 = tuple(t.data_ptr() for t in self.fp4g) if self.cfg.nvfp4 else (None,) * 3
        dm = self.cfg.dims(None if self.bias is None else self.bias.data_ptr(),
                           None if self.out16 is None else self.out16.data_ptr(), w_scales=ws, w4=w4,
                           fp4_global=g4)
        if self.norm_w is not None:
            dm.norm_weight, dm.norm_eps, dm.norm_out = self.norm_w.data_ptr(), self.norm_eps, self.xn.data_ptr()
        if self.residual is not None:
            dm.residual = self.residual.data_ptr()
        return dm

    def forward(self, stream: torch.cuda.Stream | None = None) -> torch.Tensor:
        """Enqueues one layer call on `stream` (default: torch's current stream)."""
        s = stream if stream is not None else torch.cuda.current_stream(self.device)
        a, dm = self.args(), self.dims()
        self._keep = (a, dm)
        check(lib.moe_solve_v2(ctypes.byref(a), ctypes.byref(dm), ctypes.c_void_p(s.cuda_stream)))
        return self.out

    def capture(self, stream: torch.cuda.Stream | None = None) -> "torch.cuda.CUDAGraph":
        """Records one forward() into a CUDA graph (the decode path: a replay
        costs one launch instead of the layer's ~10 kernel launches, tensor-map
        encodes and ctypes calls).  One eager call first sets up the library
        scratch and the kernels' attributes outside the capture.  The graph
        reads x and the weights from this layer's buffers, so new tokens are
        copied into `self.x` before each replay()."""
        s = stream if stream is not None else torch.cuda.Stream(self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        self.forward(s)
        s.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            self.forward(s)
        self.graph = g
        return g

    def replay(self) -> torch.Tensor:
        """Replays the captured layer on the stream it was captured on."""
        self.graph.replay()
        return self.out

    def sync_check(self, stream: torch.cuda.Stream | None = None) -> None:
        s = stream if stream is not None else torch.cuda.current_stream(self.device)
        check(lib.moe_check_device_status(ctypes.c_void_p(s.cuda_stream)))

    # -- views --------------------------------------------------------------
    def expert_rows(self) -> np.ndarray:
        """Kept rows per expert (sum over batches of counts)."""
        return self.counts.cpu().numpy().sum(axis=0)
