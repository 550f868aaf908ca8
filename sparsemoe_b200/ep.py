"""Expert parallelism: the layer sharded over P GPUs, E/P experts per GPU.

One process per GPU; torch.distributed (NCCL) carries the two all-to-all
exchanges, libsparsemoe_b200.so does all the compute:

  1. moe_stage_route        local tokens: router, top-k, capacity slots, and the
                            kept rows gathered expert-major (dense) -- the rows
                            for owner q's experts are one contiguous block
  2. all_gather             per-expert kept-row counts of every rank  [P, E]
  3. all_to_all_single      token rows to their experts' owners
  4. moe_stage_expert_ffn   owner: grouped SwiGLU GEMMs; each (sender, local
                            expert) block of the receive buffer is one GEMM row
                            group (no reorder pass), groups ordered expert-major
  5. all_to_all_single      f32 output rows back, landing in the sender's dense
                            expert-major layout
  6. moe_stage_combine      local tokens: gate-weighted sum in route order

Routing and capacity are per batch and every batch lives on one rank (each
rank routes its own batches), so drops are decided locally exactly as on one
GPU; the rows travel in f32 on the way back, so the output equals the
single-GPU layer's on the same tokens.

The planner functions below are pure (numpy) and shared with the CPU tests.
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import LayerConfig, MoEArgs, MoeDims, check, lib


# ---- planner ---------------------------------------------------------------------
def send_splits(rows_by_expert: np.ndarray, world: int) -> list[int]:
    """Rows this rank sends to each owner: its dense expert-major block of the
    owner's experts.  rows_by_expert: [E] kept rows of this rank per expert."""
    e_loc = rows_by_expert.size // world
    return [int(rows_by_expert[q * e_loc:(q + 1) * e_loc].sum()) for q in range(world)]


def recv_plan(table: np.ndarray, rank: int):
    """table: [P, E] kept rows per (sender, expert).  Returns the receive splits
    (rows from each sender) and the GEMM group table over the receive buffer:
    groups ordered (local expert j, sender s) so one expert's weights are
    reused by consecutive groups; group (j, s) starts at sender s's block
    offset plus the rows of s's earlier local experts."""
    P, E = table.shape
    e_loc = E // P
    mine = table[:, rank * e_loc:(rank + 1) * e_loc].astype(np.int64)        # [P, e_loc]
    splits = mine.sum(axis=1)
    block = np.concatenate([[0], np.cumsum(splits)[:-1]])
    within = np.concatenate([np.zeros((P, 1), np.int64), np.cumsum(mine, axis=1)[:, :-1]], axis=1)
    rows, start, expert = [], [], []
    for j in range(e_loc):
        for s in range(P):
            rows.append(int(mine[s, j]))
            start.append(int(block[s] + within[s, j]))
            expert.append(j)
    return [int(v) for v in splits], (np.array(rows, np.int32), np.array(start, np.int32),
                                      np.array(expert, np.int32))


# ---- runner ----------------------------------------------------------------------
class ExpertParallelLayer:
    """Rank-local part of an expert-parallel layer.  `cfg` is the per-rank
    workload (its batches and tokens) and the global expert count."""

    def __init__(self, cfg: LayerConfig, device, group=None):
        import torch
        import torch.distributed as dist
        self.torch, self.dist = torch, dist
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        assert cfg.num_experts % self.world == 0, "experts must divide evenly over the ranks"
        self.cfg = cfg
        self.device = torch.device(device)
        self.e_loc = cfg.num_experts // self.world
        B, N, d, f, E, k = cfg.num_batches, cfg.tokens, cfg.d_model, cfg.d_ff, cfg.num_experts, cfg.top_k
        self.cap = cfg.capacity()
        t16 = torch.bfloat16 if cfg.bf16 else torch.float16
        wt = torch.int8 if cfg.int8 else t16
        dev = self.device
        z = lambda *s, dt: torch.empty(*s, dtype=dt, device=dev)  # noqa: E731
        T = cfg.T
        rows = max(B * E * self.cap, 1)
        # routing side (all E experts, local tokens)
        self.x = z(max(T, 1), d, dt=t16)
        self.wr = z(d, E, dt=torch.float32 if cfg.router_f32 else t16)
        self.bias = None
        self.logits = z(max(T, 1), E, dt=torch.float32)
        self.idx = z(max(T, 1), k, dt=torch.int32)
        self.w = z(max(T, 1), k, dt=torch.float32)
        self.counts = z(max(B, 1), E, dt=torch.int32)
        self.token_ids = z(rows, dt=torch.int32)
        self.token_weights = z(rows, dt=torch.float32)
        self.send_x = z(rows, d, dt=wt)
        self.back_y = z(rows, d, dt=torch.float32)
        self.out = z(max(T, 1), d, dt=torch.float32)
        self.out16 = z(max(T, 1), d, dt=t16)
        # owner side (E/P experts, rows from every rank)
        self.recv_cap = max(self.world * B * self.e_loc * self.cap, 1)
        self.wg = z(self.e_loc, d, f, dt=wt)
        self.wu = z(self.e_loc, d, f, dt=wt)
        self.wd = z(self.e_loc, f, d, dt=wt)
        self.recv_x = z(self.recv_cap, d, dt=wt)
        self.h = z(self.recv_cap, f, dt=wt)
        self.recv_y = z(self.recv_cap, d, dt=torch.float32)
        self.scales = {}
        self.last_plan = None

    def load(self, inputs: dict) -> "ExpertParallelLayer":
        """inputs from make_inputs() for the FULL expert set; this rank keeps its experts."""
        torch = self.torch

        def put(dst, arr):
            arr = np.ascontiguousarray(arr)
            src = torch.from_numpy(arr.view(np.int16)).view(dst.dtype) if arr.dtype == np.uint16 \
                else torch.from_numpy(arr)
            dst.copy_(src.reshape(dst.shape))
        lo, hi = self.rank * self.e_loc, (self.rank + 1) * self.e_loc
        if self.cfg.T > 0:
            put(self.x, inputs["x"])
        put(self.wr, inputs["wr"])
        sfx = "_q" if self.cfg.int8 else ""
        put(self.wg, inputs["wg" + sfx][lo:hi])
        put(self.wu, inputs["wu" + sfx][lo:hi])
        put(self.wd, inputs["wd" + sfx][lo:hi])
        if self.cfg.int8:
            self.scales = {k: inputs[k] for k in ("s_in", "s_gate", "s_up", "s_mid", "s_down")}
        if inputs.get("bias") is not None:
            self.bias = torch.from_numpy(inputs["bias"]).to(self.device)
        return self

    def _route_args(self) -> MoEArgs:
        a = MoEArgs()
        p = lambda t: t.data_ptr()  # noqa: E731
        a.input, a.router_weights, a.expert_logits = p(self.x), p(self.wr), p(self.logits)
        a.selected_expert_indices, a.selected_expert_weights = p(self.idx), p(self.w)
        a.expert_counts, a.expert_token_ids, a.expert_token_weights = p(self.counts), p(self.token_ids), \
            p(self.token_weights)
        if self.cfg.int8:
            a.per_expert_wmma_inputs_int8 = p(self.send_x)
            self._scales_into(a)
        else:
            a.per_expert_wmma_inputs = p(self.send_x)
        a.hidden_mlp_layer_2_out = p(self.back_y)
        a.final_output = p(self.out)
        a.num_batches = self.cfg.num_batches
        a.use_capacity = self.cfg.cap >= 0
        a.cap = self.cap
        return a

    def _ffn_args(self) -> MoEArgs:
        a = MoEArgs()
        p = lambda t: t.data_ptr()  # noqa: E731
        if self.cfg.int8:
            a.expert_gate_proj_weights_int8, a.expert_up_proj_weights_int8 = p(self.wg), p(self.wu)
            a.expert_down_proj_weights_int8 = p(self.wd)
            a.per_expert_wmma_inputs_int8, a.hidden_mlp_layer_1_out_int8 = p(self.recv_x), p(self.h)
            self._scales_into(a)
        else:
            a.expert_gate_proj_weights, a.expert_up_proj_weights = p(self.wg), p(self.wu)
            a.expert_down_proj_weights = p(self.wd)
            a.per_expert_wmma_inputs, a.hidden_mlp_layer_1_out_fp16 = p(self.recv_x), p(self.h)
        a.hidden_mlp_layer_2_out = p(self.recv_y)
        return a

    def _scales_into(self, a):
        sc = self.scales
        a.scale_input_act, a.scale_gate_w, a.scale_up_w = sc["s_in"], sc["s_gate"], sc["s_up"]
        a.scale_mid_act, a.scale_down_w = sc["s_mid"], sc["s_down"]

    PHASES = ("route", "dispatch_a2a", "expert_ffn", "return_a2a", "combine")

    def forward(self, stream=None, events=None):
        """One layer call.  `events` (6 torch.cuda.Event, optional) are recorded
        on the stream around the phases in PHASES order."""
        torch, dist = self.torch, self.dist
        cfg = self.cfg
        s = stream if stream is not None else torch.cuda.current_stream(self.device)
        sp = ctypes.c_void_p(s.cuda_stream)
        mark = (lambda i: events[i].record(s)) if events is not None else (lambda i: None)
        mark(0)
        dims = cfg.dims(None if self.bias is None else self.bias.data_ptr(), self.out16.data_ptr())
        ra = self._route_args()
        check(lib.moe_stage_route(ctypes.byref(ra), ctypes.byref(dims), sp))
        mark(1)
        # 2. kept rows per expert of every rank
        mine = self.counts[: cfg.num_batches].sum(dim=0, dtype=torch.int32) if cfg.num_batches > 0 else \
            torch.zeros(cfg.num_experts, dtype=torch.int32, device=self.device)
        table = torch.empty(self.world, cfg.num_experts, dtype=torch.int32, device=self.device)
        dist.all_gather_into_tensor(table, mine, group=self.group)
        table_h = table.cpu().numpy()                         # host needs the split sizes
        ssplit = send_splits(table_h[self.rank], self.world)
        rsplit, (g_rows, g_start, g_exp) = recv_plan(table_h, self.rank)
        n_send, n_recv = sum(ssplit), sum(rsplit)
        # 3. rows to their owners
        dist.all_to_all_single(self.recv_x[:n_recv], self.send_x[:n_send], rsplit, ssplit, group=self.group)
        mark(2)
        # 4. owner FFN
        fa = self._ffn_args()
        fdims = MoeDims(0, 0, cfg.d_model, cfg.d_ff, self.e_loc, 1, cfg.capacity_factor, 0, cfg.dtype, 0, None,
                        None)
        check(lib.moe_stage_expert_ffn(ctypes.byref(fa), ctypes.byref(fdims), g_rows.ctypes.data,
                                       g_start.ctypes.data, g_exp.ctypes.data, len(g_rows), self.recv_cap, sp))
        mark(3)
        # 5. outputs back
        dist.all_to_all_single(self.back_y[:n_send], self.recv_y[:n_recv], ssplit, rsplit, group=self.group)
        mark(4)
        # 6. combine
        check(lib.moe_stage_combine(ctypes.byref(ra), ctypes.byref(dims), sp))
        mark(5)
        self._keep = (ra, fa, dims, fdims, g_rows, g_start, g_exp)
        self.last_plan = {"send": ssplit, "recv": rsplit, "table": table_h, "owner_rows": int(n_recv)}
        return self.out

    def sync_check(self, stream=None):
        s = stream if stream is not None else self.torch.cuda.current_stream(self.device)
        check(lib.moe_check_device_status(ctypes.c_void_p(s.cuda_stream)))
