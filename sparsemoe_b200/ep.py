"""Expert parallelism: the layer sharded over P GPUs, E/P experts per GPU.

One process per GPU; torch.distributed (NCCL) carries the two all-to-all
exchanges, libsparsemoe_b200.so does all the compute:

  1. moe_stage_route        local tokens: router, top-k, capacity slots, and the
                            kept rows gathered expert-major (dense) -- the rows
                            for owner q's experts are one contiguous block
  2. all_gather             per-expert kept-row counts of every rank  [P, E]
  3. all_to_all_single      token rows to their experts' owners (second stream)
  4. moe_stage_expert_ffn   owner: grouped SwiGLU GEMMs; each (sender, local
                            expert) block of the receive buffer is one GEMM row
                            group (no reorder pass), groups ordered expert-major
  5. all_to_all_single      f32 output rows back, landing in the sender's dense
                            expert-major layout (second stream)
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
class _Chunk:
    """One group of whole batches routed, exchanged and combined together."""


class ExpertParallelLayer:
    """Rank-local part of an expert-parallel layer.  `cfg` is the per-rank
    workload (its batches and tokens) and the global expert count.

    The rank's batches can be split into `chunks` groups that pipeline: while
    the owner GEMMs run on chunk c (compute stream), chunk c+1's rows arrive
    and chunk c-1's outputs return on a second stream (NCCL all-to-all).  Each
    chunk has its own routing-table scratch (MoeDims.scratch).  Default 1:
    measured on 2 B200s (Mixtral shape), 2 chunks were slower (11.4 vs 10.6
    ms) because NCCL's kernels take SMs from the persistent GEMM and the
    weights are streamed once per chunk."""

    PHASES = ("route", "exchange_and_ffn", "combine")

    def __init__(self, cfg: LayerConfig, device, group=None, chunks: int | None = None):
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
        if chunks is None:
            chunks = 1
        assert B % chunks == 0 or B == 0, "chunks must divide num_batches"
        self.n_chunks = max(chunks, 1)
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
        # chunk views and scratch
        Bc = B // self.n_chunks if B else 0
        self.chunk_cfg = LayerConfig(Bc, N, d, f, E, k, cfg.capacity_factor, cfg.dtype, cfg.router_f32, cfg.zipf_s,
                                     cfg.cap, cfg.act_scale, cfg.mid_scale)
        sdims = self.chunk_cfg.dims()
        ws_bytes = int(lib.moe_workspace_bytes(ctypes.byref(sdims)))
        ws_bytes = max(ws_bytes, 1 << 16)
        self.chunks = []
        Tc, rc, ocap = Bc * N, Bc * E * self.cap, self.world * Bc * self.e_loc * self.cap
        for c in range(self.n_chunks):
            ch = _Chunk()
            t0, r0, o0 = c * Tc, c * rc, c * ocap
            ch.x, ch.logits, ch.idx, ch.w = self.x[t0:t0 + Tc], self.logits[t0:t0 + Tc], self.idx[t0:t0 + Tc], \
                self.w[t0:t0 + Tc]
            ch.counts = self.counts[c * Bc:(c + 1) * Bc]
            ch.token_ids, ch.token_weights = self.token_ids[r0:r0 + rc], self.token_weights[r0:r0 + rc]
            ch.send_x, ch.back_y = self.send_x[r0:r0 + rc], self.back_y[r0:r0 + rc]
            ch.out, ch.out16 = self.out[t0:t0 + Tc], self.out16[t0:t0 + Tc]
            ch.recv_x, ch.h, ch.recv_y = self.recv_x[o0:o0 + ocap], self.h[o0:o0 + ocap], self.recv_y[o0:o0 + ocap]
            ch.recv_cap = ocap
            ch.scratch = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
            ch.ffn_scratch = torch.empty(1 << 16, dtype=torch.uint8, device=dev)
            self.chunks.append(ch)
        self.comm_stream = torch.cuda.Stream(device=dev)

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

    def _scales_into(self, a):
        sc = self.scales
        a.scale_input_act, a.scale_gate_w, a.scale_up_w = sc["s_in"], sc["s_gate"], sc["s_up"]
        a.scale_mid_act, a.scale_down_w = sc["s_mid"], sc["s_down"]

    def _route_args(self, ch) -> MoEArgs:
        a = MoEArgs()
        p = lambda t: t.data_ptr()  # noqa: E731
        a.input, a.router_weights, a.expert_logits = p(ch.x), p(self.wr), p(ch.logits)
        a.selected_expert_indices, a.selected_expert_weights = p(ch.idx), p(ch.w)
        a.expert_counts, a.expert_token_ids, a.expert_token_weights = p(ch.counts), p(ch.token_ids), \
            p(ch.token_weights)
        if self.cfg.int8:
            a.per_expert_wmma_inputs_int8 = p(ch.send_x)
            self._scales_into(a)
        else:
            a.per_expert_wmma_inputs = p(ch.send_x)
        a.hidden_mlp_layer_2_out = p(ch.back_y)
        a.final_output = p(ch.out)
        a.num_batches = self.chunk_cfg.num_batches
        a.use_capacity = self.cfg.cap >= 0
        a.cap = self.cap
        return a

    def _ffn_args(self, ch) -> MoEArgs:
        a = MoEArgs()
        p = lambda t: t.data_ptr()  # noqa: E731
        if self.cfg.int8:
            a.expert_gate_proj_weights_int8, a.expert_up_proj_weights_int8 = p(self.wg), p(self.wu)
            a.expert_down_proj_weights_int8 = p(self.wd)
            a.per_expert_wmma_inputs_int8, a.hidden_mlp_layer_1_out_int8 = p(ch.recv_x), p(ch.h)
            self._scales_into(a)
        else:
            a.expert_gate_proj_weights, a.expert_up_proj_weights = p(self.wg), p(self.wu)
            a.expert_down_proj_weights = p(self.wd)
            a.per_expert_wmma_inputs, a.hidden_mlp_layer_1_out_fp16 = p(ch.recv_x), p(ch.h)
        a.hidden_mlp_layer_2_out = p(ch.recv_y)
        return a

    def forward(self, stream=None, timing=None):
        """One layer call.  `timing` (optional dict) receives torch.cuda.Event
        lists: 'start', 'routed', 'ffn' (pairs per chunk), 'combine', 'end'."""
        torch, dist = self.torch, self.dist
        cfg = self.cfg
        S = stream if stream is not None else torch.cuda.current_stream(self.device)
        C = self.comm_stream
        sp = ctypes.c_void_p(S.cuda_stream)

        def ev(name):
            if timing is None:
                return
            e = torch.cuda.Event(enable_timing=True)
            e.record(S)
            timing.setdefault(name, []).append(e)
        ev("start")
        keep = []
        bias = None if self.bias is None else self.bias.data_ptr()
        for ch in self.chunks:                                   # 1. route every chunk
            ch.dims = self.chunk_cfg.dims(bias, ch.out16.data_ptr(), ch.scratch.data_ptr(), ch.scratch.numel())
            ch.ra = self._route_args(ch)
            check(lib.moe_stage_route(ctypes.byref(ch.ra), ctypes.byref(ch.dims), sp))
        ev("routed")
        nc = self.n_chunks
        mine = self.counts[: cfg.num_batches].view(nc, -1, cfg.num_experts).sum(dim=1, dtype=torch.int32)
        table = torch.empty(self.world, nc, cfg.num_experts, dtype=torch.int32, device=self.device)
        dist.all_gather_into_tensor(table, mine.contiguous(), group=self.group)   # 2. [P, chunk, E]
        table_h = table.cpu().numpy()                      # the host needs the split sizes
        routed = torch.cuda.Event()
        routed.record(S)
        plans = []
        for c, ch in enumerate(self.chunks):
            ss = send_splits(table_h[self.rank, c], self.world)
            rs, groups = recv_plan(table_h[:, c], self.rank)
            plans.append((ss, rs, groups))
        sends = []
        with torch.cuda.stream(C):                          # 3. rows to owners, all chunks
            C.wait_event(routed)
            for ch, (ss, rs, _) in zip(self.chunks, plans):
                sends.append(dist.all_to_all_single(ch.recv_x[:sum(rs)], ch.send_x[:sum(ss)], rs, ss,
                                                    group=self.group, async_op=True))
        rets = []
        fdims = MoeDims(0, 0, cfg.d_model, cfg.d_ff, self.e_loc, 1, cfg.capacity_factor, 0, cfg.dtype, 0, None,
                        None, None, 0)
        for ch, (ss, rs, (g_rows, g_start, g_exp)), work in zip(self.chunks, plans, sends):
            work.wait()                                      # compute stream waits for chunk's rows
            ev("ffn")
            fa = self._ffn_args(ch)
            fd = MoeDims(*[getattr(fdims, n) for n, _ in MoeDims._fields_])
            fd.scratch, fd.scratch_bytes = ch.ffn_scratch.data_ptr(), ch.ffn_scratch.numel()
            check(lib.moe_stage_expert_ffn(ctypes.byref(fa), ctypes.byref(fd), g_rows.ctypes.data,
                                           g_start.ctypes.data, g_exp.ctypes.data, len(g_rows), ch.recv_cap, sp))
            ev("ffn")
            done = torch.cuda.Event()
            done.record(S)
            with torch.cuda.stream(C):                      # 5. this chunk's outputs back
                C.wait_event(done)
                rets.append(dist.all_to_all_single(ch.back_y[:sum(ss)], ch.recv_y[:sum(rs)], ss, rs,
                                                   group=self.group, async_op=True))
            keep.append((fa, fd, g_rows, g_start, g_exp))
        for ch, work in zip(self.chunks, rets):             # 6. combine
            work.wait()
            ev("combine")
            check(lib.moe_stage_combine(ctypes.byref(ch.ra), ctypes.byref(ch.dims), sp))
        ev("end")
        self._keep = keep
        self.last_plan = {"table": table_h, "owner_rows": int(sum(sum(p[1]) for p in plans))}
        return self.out

    def sync_check(self, stream=None):
        """Synchronises and raises if any chunk's kernels reported a device-side
        wait timeout (the status word heads every scratch block)."""
        from . import MOE_ERR_TIMEOUT, MoeError
        s = stream if stream is not None else self.torch.cuda.current_stream(self.device)
        check(lib.moe_check_device_status(ctypes.c_void_p(s.cuda_stream)))
        for c, ch in enumerate(self.chunks):
            for buf in (ch.scratch, ch.ffn_scratch):
                word = int(buf[:4].view(self.torch.int32).item())
                if word != 0:
                    raise MoeError(MOE_ERR_TIMEOUT, f"chunk {c}: device-side wait timed out (status {word})")
