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

Two ways to place the tokens:

* per-rank batches (default): every batch lives on one rank, so capacity and
  drops are decided locally exactly as on one GPU;
* global batches (`global_batch=True`): every batch of world*N tokens is split
  over the ranks in token order (rank r holds tokens [r*N, (r+1)*N)); CAP is
  that of the whole batch and a route is kept iff its slot in global route-id
  order is < CAP.  Step 1 then runs in two phases: router + per-(batch,
  expert) route totals (moe_stage_route_counts), an all_gather of the totals,
  and the slots with each rank's prefix over the lower ranks' totals as
  slot_base (moe_stage_route_finish).

The rows travel back in f32, so the output equals the single-GPU layer's on
the same tokens.

Transport: NCCL all-to-all (rows and results on a second stream), or
(transport="peer") NVLink peer memory with no host synchronisation -- the
kept-row table is all-gathered on the device, moe_ep_plan places every row,
the gather writes each row into its owner's receive buffer, and the owner's
down-GEMM epilogue stores each result row into its sender's buffer.  With the
peer transport the experts can be owned strided (placement="strided": rank q
holds experts q, q+P, ...), which spreads a popularity skew over low expert
indices (the Zipf-biased routers) across the ranks.  All weight formats run: 16-bit, per-tensor int8, 4-bit
(INT4 g128, NVFP4) with bf16 rows on the wire, and the dynamically quantised
FP8-block / int8-per-channel formats, whose 8-bit rows travel with their row
scales (a second all-to-all of [rows, d/128] or [rows] f32).

The planner functions below are pure (numpy) and shared with the CPU tests.
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import LayerConfig, MoEArgs, MoeDims, capacity, check, lib


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


def ep_plan_host(table: np.ndarray, rank: int, strided: bool = False) -> np.ndarray:
    """Host restatement of moe_ep_plan (the device plan of the peer transport)
    for one rank: table [P, E] kept rows per (sender, expert).  Returns the
    7*E int32 plan: owner[E] | row0[E] | g_rows | g_start | g_expert |
    g_sender | g_out_row (G = E groups, g = j * P + s)."""
    P, E = table.shape
    el = E // P
    t = table.astype(np.int64)

    def gexp(q, j):
        return j * P + q if strided else q * el + j
    to_owner = np.array([[sum(t[s, gexp(q, j)] for j in range(el)) for q in range(P)] for s in range(P)])
    recv_off = np.concatenate([np.zeros((1, P), np.int64), np.cumsum(to_owner, axis=0)[:-1]], axis=0)
    plan = np.zeros(7 * E, np.int64)
    for e in range(E):
        q, lj = (e % P, e // P) if strided else (e // el, e % el)
        plan[e] = q
        plan[E + e] = recv_off[rank, q] + sum(t[rank, gexp(q, j2)] for j2 in range(lj))
    for g in range(E):
        j, s = divmod(g, P)
        ge = gexp(rank, j)
        within = sum(t[s, gexp(rank, j2)] for j2 in range(j))
        plan[2 * E + g] = t[s, ge]
        plan[3 * E + g] = recv_off[s, rank] + within
        plan[4 * E + g] = j
        plan[5 * E + g] = s
        plan[6 * E + g] = t[s, :ge].sum()
    return plan.astype(np.int32)


# ---- runner ----------------------------------------------------------------------
class _Ptr:
    """A raw device address with the data_ptr() of a tensor."""

    def __init__(self, addr: int):
        self.addr = addr

    def data_ptr(self) -> int:
        return self.addr


class _Chunk:
    """One group of whole batches routed, exchanged and combined together."""


def _fmt(cfg: LayerConfig):
    """(wire dtype of the A rows, dtype of h, activation scales per row) of a format."""
    import torch
    t16 = torch.bfloat16 if cfg.act_bf16 else torch.float16
    if cfg.int8 or cfg.int8ch:
        return torch.int8, torch.int8, (1 if cfg.int8ch else 0)
    if cfg.fp8:
        return torch.uint8, torch.uint8, cfg.d_model // 128
    return t16, t16, 0


class ExpertParallelLayer:
    """Rank-local part of an expert-parallel layer.  `cfg` is the per-rank
    workload (its batches and tokens -- with `global_batch`, its shard of
    every batch) and the global expert count.

    The rank's batches can be split into `chunks` groups that pipeline: while
    the owner GEMMs run on chunk c (compute stream), chunk c+1's rows arrive
    and chunk c-1's outputs return on a second stream (NCCL all-to-all).  Each
    chunk has its own routing-table scratch (MoeDims.scratch).  Default 1:
    measured on 2 B200s (Mixtral shape), 2 chunks were slower (11.4 vs 10.6
    ms) because NCCL's kernels take SMs from the persistent GEMM and the
    weights are streamed once per chunk.

    With `health_timeout` (seconds) every forward() first runs a host-side
    liveness barrier (health.PeerWatch over the process group's store): a
    peer that left between steps raises health.PeerLost on the survivors
    before any kernel or collective of the step is enqueued."""

    PHASES = ("route", "exchange_and_ffn", "combine")

    def __init__(self, cfg: LayerConfig, device, group=None, chunks: int | None = None,
                 global_batch: bool = False, transport: str = "nccl", placement: str = "contiguous",
                 health_timeout: float | None = None, store=None):
        import torch
        import torch.distributed as dist
        self.torch, self.dist = torch, dist
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        assert cfg.num_experts % self.world == 0, "experts must divide evenly over the ranks"
        assert not (cfg.int4ptx or cfg.fp8pt), \
            "the reference's packed int4 and per-tensor fp8 formats run on one GPU (solve / moe_solve_v2)"
        self.cfg = cfg
        self.global_batch = global_batch
        self.device = torch.device(device)
        self.e_loc = cfg.num_experts // self.world
        B, N, d, f, E, k = cfg.num_batches, cfg.tokens, cfg.d_model, cfg.d_ff, cfg.num_experts, cfg.top_k
        chunks = 1 if chunks is None else chunks
        assert B % chunks == 0 or B == 0, "chunks must divide num_batches"
        assert not (global_batch and chunks > 1), "global batches run as one chunk"
        assert transport in ("nccl", "peer"), transport
        assert not (transport == "peer" and chunks > 1), "the peer transport runs as one chunk"
        self.transport = transport
        assert placement in ("contiguous", "strided"), placement
        assert not (placement == "strided" and transport != "peer"), "strided placement needs the peer transport"
        self.placement = placement
        self.n_chunks = max(chunks, 1)
        if global_batch:
            # CAP of the whole batch (world shards of N tokens); cap < 0: no drop
            if cfg.cap > 0:
                self.cap = cfg.cap
            elif cfg.cap < 0:
                self.cap = N * self.world
            else:
                self.cap = capacity(N * self.world, k, E, cfg.capacity_factor)
        else:
            self.cap = cfg.capacity()
        t16 = torch.bfloat16 if cfg.act_bf16 else torch.float16
        at, ht, self.n_scale = _fmt(cfg)
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
        self.send_x = z(rows, d, dt=at)
        self.send_scale = z(rows, self.n_scale, dt=torch.float32) if self.n_scale else None
        self.back_y = z(rows, d, dt=torch.float32)
        self.out = z(max(T, 1), d, dt=torch.float32)
        self.out16 = z(max(T, 1), d, dt=t16)
        self.raw = z(max(B, 1), E, dt=torch.int32) if global_batch else None
        self.slot_base = z(max(B, 1), E, dt=torch.int32) if global_batch else None
        # owner side (E/P experts, rows from every rank): per (batch, local
        # expert) at most CAP rows in all -- per sender with per-rank batches
        per_owner = B * self.e_loc * self.cap
        self.recv_cap = max(per_owner if global_batch else self.world * per_owner, 1)
        self.recv_x = z(self.recv_cap, d, dt=at)
        self.recv_scale = z(self.recv_cap, self.n_scale, dt=torch.float32) if self.n_scale else None
        self.h = z(self.recv_cap, f, dt=ht)
        self.recv_y = z(self.recv_cap, d, dt=torch.float32)
        self.weights = {}
        self.scales = {}
        self.last_plan = None
        # chunk views and scratch
        Bc = B // self.n_chunks if B else 0
        self.chunk_cfg = LayerConfig(Bc, N, d, f, E, k, cfg.capacity_factor, cfg.dtype, cfg.router_f32, cfg.zipf_s,
                                     self.cap if global_batch else cfg.cap, cfg.act_scale, cfg.mid_scale)
        sdims = self.chunk_cfg.dims()
        ws_bytes = max(int(lib.moe_workspace_bytes(ctypes.byref(sdims))), 1 << 16)
        self.chunks = []
        Tc, rc, ocap = Bc * N, Bc * E * self.cap, self.recv_cap // self.n_chunks
        fdims = self._ffn_dims_base()
        ffn_bytes = max(int(lib.moe_ffn_scratch_bytes(ctypes.byref(fdims), ocap)), 1 << 16)
        for c in range(self.n_chunks):
            ch = _Chunk()
            t0, r0, o0 = c * Tc, c * rc, c * ocap
            ch.x, ch.logits, ch.idx, ch.w = self.x[t0:t0 + Tc], self.logits[t0:t0 + Tc], self.idx[t0:t0 + Tc], \
                self.w[t0:t0 + Tc]
            ch.counts = self.counts[c * Bc:(c + 1) * Bc]
            ch.token_ids, ch.token_weights = self.token_ids[r0:r0 + rc], self.token_weights[r0:r0 + rc]
            ch.send_x, ch.back_y = self.send_x[r0:r0 + rc], self.back_y[r0:r0 + rc]
            ch.send_scale = self.send_scale[r0:r0 + rc] if self.n_scale else None
            ch.out, ch.out16 = self.out[t0:t0 + Tc], self.out16[t0:t0 + Tc]
            ch.recv_x, ch.h, ch.recv_y = self.recv_x[o0:o0 + ocap], self.h[o0:o0 + ocap], self.recv_y[o0:o0 + ocap]
            ch.recv_scale = self.recv_scale[o0:o0 + ocap] if self.n_scale else None
            ch.recv_cap = ocap
            ch.scratch = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
            ch.ffn_scratch = torch.empty(ffn_bytes, dtype=torch.uint8, device=dev)
            self.chunks.append(ch)
        self.comm_stream = torch.cuda.Stream(device=dev)
        # host-side liveness check before every call (health_timeout seconds per step)
        self.watch = None
        if health_timeout is not None:
            from .health import PeerWatch
            self.watch = PeerWatch(store if store is not None else PeerWatch.default_store(), self.rank,
                                   self.world, health_timeout)
        if transport == "peer":
            self._setup_peer()

    # -- peer memory (transport="peer") ---------------------------------------------
    def _setup_peer(self):
        """Receive buffers (rows, row scales) and return buffers (f32 rows)
        that the other ranks map through CUDA IPC: the senders' dispatch (row scatter) kernels
        store their rows straight into the owners' receive buffers, and owners' down-GEMM
        epilogues store result rows straight into the senders' return
        buffers."""
        torch, dist = self.torch, self.dist
        cfg, d = self.cfg, self.cfg.d_model
        ch = self.chunks[0]
        self._row_bytes = d * self.recv_x.element_size()
        self._scale_bytes = 4 * self.n_scale
        sizes = {"recv_x": self.recv_cap * self._row_bytes, "back_y": ch.send_x.shape[0] * d * 4}
        if self.n_scale:
            sizes["recv_scale"] = self.recv_cap * self._scale_bytes
        self.peer_local, self.peer_maps = {}, {}
        for name, nbytes in sizes.items():
            ptr, handle = ctypes.c_void_p(), (ctypes.c_ubyte * 64)()
            check(lib.moe_peer_alloc(max(nbytes, 256), ctypes.byref(ptr), handle))
            self.peer_local[name] = ptr.value
            mine = torch.tensor(list(bytes(handle)), dtype=torch.uint8, device=self.device)
            every = torch.empty(self.world, 64, dtype=torch.uint8, device=self.device)
            dist.all_gather_into_tensor(every, mine, group=self.group)
            every = every.cpu().numpy()
            maps = []
            for r in range(self.world):
                if r == self.rank:
                    maps.append(ptr.value)
                    continue
                h = (ctypes.c_ubyte * 64)(*every[r].tolist())
                q = ctypes.c_void_p()
                check(lib.moe_peer_open(h, ctypes.byref(q)))
                maps.append(q.value)
            self.peer_maps[name] = maps
        self._bar = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.table = torch.zeros(self.world, cfg.num_experts, dtype=torch.int32, device=self.device)
        self.plan = torch.zeros(7 * cfg.num_experts, dtype=torch.int32, device=self.device)

    def close(self):
        """Unmaps the peers' buffers and frees this rank's (peer transport)."""
        if getattr(self, "peer_maps", None):
            self.torch.cuda.synchronize(self.device)
            for maps in self.peer_maps.values():
                for r, ptr in enumerate(maps):
                    if r != self.rank:
                        lib.moe_peer_close(ctypes.c_void_p(ptr))
            for ptr in self.peer_local.values():
                lib.moe_peer_free(ctypes.c_void_p(ptr))
            self.peer_maps, self.peer_local = {}, {}

    def _barrier(self, S):
        with self.torch.cuda.stream(S):
            self.dist.all_reduce(self._bar, group=self.group)

    # -- weights ------------------------------------------------------------------
    def load(self, inputs: dict, local: bool = False) -> "ExpertParallelLayer":
        """inputs from make_inputs(): x (this rank's tokens), wr, bias and the
        weights of the FULL expert set (this rank keeps its E/P experts), or
        with local=True weights that already hold only this rank's experts."""
        torch, cfg = self.torch, self.cfg

        def dev_t(arr):
            arr = np.ascontiguousarray(arr)
            t = torch.from_numpy(arr.view(np.int16)) if arr.dtype == np.uint16 else torch.from_numpy(arr)
            return t.to(self.device)

        def mine(arr):
            if local:
                return arr
            if self.placement == "strided":
                return np.ascontiguousarray(arr[self.rank::self.world])
            return arr[self.rank * self.e_loc:(self.rank + 1) * self.e_loc]
        if cfg.T > 0:
            x = dev_t(inputs["x"])
            self.x[: cfg.T].copy_(x.view(self.x.dtype).reshape(cfg.T, cfg.d_model))
        wr = dev_t(inputs["wr"])
        self.wr.copy_(wr.view(self.wr.dtype).reshape(self.wr.shape))
        quant = cfg.int8 or cfg.int8ch or cfg.fp8 or cfg.w4
        sfx = "_q" if quant else ""
        t16 = self.x.dtype
        for n in ("wg", "wu", "wd"):
            t = dev_t(mine(inputs[n + sfx]))
            self.weights[n] = t.view(t16) if not quant else t
        if cfg.int8:
            self.scales = {k: inputs[k] for k in ("s_in", "s_gate", "s_up", "s_mid", "s_down")}
        if cfg.channel_scaled:
            self.weights["w_scale"] = [dev_t(mine(inputs[k])) for k in ("sg", "su", "sd")]
        if cfg.w4:
            keys = ("wg_s", "wu_s", "wd_s") + (() if cfg.nvfp4 else ("wg_z", "wu_z", "wd_z"))
            self.weights["w4"] = [dev_t(mine(inputs[k])) for k in keys]
            if cfg.nvfp4:
                self.weights["fp4g"] = [dev_t(mine(np.asarray(inputs[k], np.float32)))
                                        for k in ("wg_g", "wu_g", "wd_g")]
        if inputs.get("bias") is not None:
            self.bias = torch.from_numpy(inputs["bias"]).to(self.device)
        return self

    @property
    def wg(self):
        return self.weights["wg"]

    @property
    def wu(self):
        return self.weights["wu"]

    @property
    def wd(self):
        return self.weights["wd"]

    # -- call arguments -------------------------------------------------------------
    def _scales_into(self, a):
        sc = self.scales
        a.scale_input_act, a.scale_gate_w, a.scale_up_w = sc["s_in"], sc["s_gate"], sc["s_up"]
        a.scale_mid_act, a.scale_down_w = sc["s_mid"], sc["s_down"]

    def _set_rows(self, a, rows, h=None):
        cfg, p = self.cfg, (lambda t: t.data_ptr())
        if cfg.int8 or cfg.int8ch:
            a.per_expert_wmma_inputs_int8 = p(rows)
            if h is not None:
                a.hidden_mlp_layer_1_out_int8 = p(h)
            if cfg.int8:
                self._scales_into(a)
        elif cfg.fp8:
            a.per_expert_wmma_inputs_fp8 = p(rows)
            if h is not None:
                a.hidden_mlp_layer_1_out_fp8 = p(h)
        else:
            a.per_expert_wmma_inputs = p(rows)
            if h is not None:
                a.hidden_mlp_layer_1_out_fp16 = p(h)

    def _route_args(self, ch) -> MoEArgs:
        a = MoEArgs()
        p = lambda t: t.data_ptr()  # noqa: E731
        a.input, a.router_weights, a.expert_logits = p(ch.x), p(self.wr), p(ch.logits)
        a.selected_expert_indices, a.selected_expert_weights = p(ch.idx), p(ch.w)
        a.expert_counts, a.expert_token_ids, a.expert_token_weights = p(ch.counts), p(ch.token_ids), \
            p(ch.token_weights)
        self._set_rows(a, ch.send_x)
        a.hidden_mlp_layer_2_out = p(ch.back_y)
        a.final_output = p(ch.out)
        a.num_batches = self.chunk_cfg.num_batches
        a.use_capacity = self.cfg.cap >= 0
        a.cap = self.cap
        return a

    def _ffn_args(self, ch) -> MoEArgs:
        cfg, a = self.cfg, MoEArgs()
        p = lambda t: t.data_ptr()  # noqa: E731
        wg, wu, wd = p(self.wg), p(self.wu), p(self.wd)
        if cfg.int8 or cfg.int8ch:
            a.expert_gate_proj_weights_int8, a.expert_up_proj_weights_int8, a.expert_down_proj_weights_int8 = \
                wg, wu, wd
        elif cfg.fp8:
            a.expert_gate_proj_weights_fp8, a.expert_up_proj_weights_fp8, a.expert_down_proj_weights_fp8 = \
                wg, wu, wd
        elif cfg.w4:
            a.expert_gate_proj_weights_int4, a.expert_up_proj_weights_int4, a.expert_down_proj_weights_int4 = \
                wg, wu, wd
        else:
            a.expert_gate_proj_weights, a.expert_up_proj_weights, a.expert_down_proj_weights = wg, wu, wd
        self._set_rows(a, ch.recv_x, ch.h)
        a.hidden_mlp_layer_2_out = p(ch.recv_y)
        return a

    def _ffn_dims_base(self) -> MoeDims:
        cfg = self.cfg
        fd = MoeDims(0, 0, cfg.d_model, cfg.d_ff, self.e_loc, 1, cfg.capacity_factor, 0, cfg.dtype, 0)
        if self.weights.get("w_scale"):
            fd.w_scale_gate, fd.w_scale_up, fd.w_scale_down = (t.data_ptr() for t in self.weights["w_scale"])
        if self.weights.get("w4"):
            w4 = [t.data_ptr() for t in self.weights["w4"]]
            fd.w4_scale_gate, fd.w4_scale_up, fd.w4_scale_down = w4[:3]
            if len(w4) == 6:
                fd.w4_zero_gate, fd.w4_zero_up, fd.w4_zero_down = w4[3:]
        if self.weights.get("fp4g"):
            fd.fp4_global_gate, fd.fp4_global_up, fd.fp4_global_down = (t.data_ptr() for t in self.weights["fp4g"])
        return fd

    # -- one layer call -------------------------------------------------------------
    def _forward_peer(self, S, ev):
        """Steps 2-5 over peer memory with no host synchronisation: the
        kept-row table is all-gathered on the device, moe_ep_plan turns it into
        this rank's destinations and owner row groups, the gather writes each
        row straight into its owner's receive buffer, and after a barrier the
        owner FFN's down-GEMM epilogue stores the results into the senders'
        return buffers; a second barrier orders the combine."""
        torch, cfg = self.torch, self.cfg
        ch = self.chunks[0]
        sp = ctypes.c_void_p(S.cuda_stream)
        P, E = self.world, cfg.num_experts
        mine = self.counts[: cfg.num_batches].sum(dim=0, dtype=torch.int32)
        with torch.cuda.stream(S):
            self.dist.all_gather_into_tensor(self.table, mine, group=self.group)
        check(lib.moe_ep_plan(ctypes.c_void_p(self.table.data_ptr()), P, self.rank, E,
                              int(self.placement == "strided"), ctypes.c_void_p(self.plan.data_ptr()), sp))
        rows = (ctypes.c_void_p * P)(*self.peer_maps["recv_x"])
        scales = (ctypes.c_void_p * P)(*self.peer_maps["recv_scale"]) if self.n_scale else None
        ev("dispatch")
        check(lib.moe_stage_dispatch_peer(ctypes.byref(ch.ra), ctypes.byref(ch.dims),
                                          ctypes.c_void_p(self.plan.data_ptr()), rows, scales, P, sp))
        ev("dispatch")
        self._barrier(S)
        ev("ffn")
        fa = self._ffn_args(ch)
        fa.per_expert_wmma_inputs = fa.per_expert_wmma_inputs_int8 = fa.per_expert_wmma_inputs_fp8 = None
        self._set_rows(fa, _Ptr(self.peer_local["recv_x"]), ch.h)
        fd = self._ffn_dims_base()
        fd.scratch, fd.scratch_bytes = ch.ffn_scratch.data_ptr(), ch.ffn_scratch.numel()
        if self.n_scale:
            fd.act_scale = self.peer_local["recv_scale"]
        bases = (ctypes.c_void_p * P)(*self.peer_maps["back_y"])
        check(lib.moe_stage_expert_ffn_planned(ctypes.byref(fa), ctypes.byref(fd),
                                               ctypes.c_void_p(self.plan.data_ptr()), E, self.recv_cap, bases, P, sp))
        ev("ffn")
        self._barrier(S)
        self._keep = (fa, fd, rows, scales, bases)

    def owner_rows(self) -> int:
        """Rows this rank's experts processed in the last call (synchronises)."""
        if self.transport == "peer":
            t = self.table.cpu().numpy()
            if self.placement == "strided":
                return int(t[:, self.rank::self.world].sum())
            return int(t[:, self.rank * self.e_loc:(self.rank + 1) * self.e_loc].sum())
        return self.last_plan["owner_rows"]

    def forward(self, stream=None, timing=None):
        """One layer call.  `timing` (optional dict) receives torch.cuda.Event
        lists: 'start', 'routed', 'ffn' (pairs per chunk), 'combine', 'end'
        (and, peer transport, 'dispatch': the peer gather's start and end)."""
        torch = self.torch
        if self.watch is not None:
            self.watch.step()      # raises PeerLost before anything of this call is enqueued
        S = stream if stream is not None else torch.cuda.current_stream(self.device)
        # every torch op and collective below (all_gather of the route totals
        # and kept-row table, the slot-base and count sums) then runs on S, in
        # order with the library kernels enqueued on S
        with torch.cuda.stream(S):
            return self._forward(S, timing)

    def _forward(self, S, timing):
        torch, dist = self.torch, self.dist
        cfg = self.cfg
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
            if self.n_scale:
                ch.dims.act_scale = ch.send_scale.data_ptr()
            ch.dims.skip_gather = 1 if self.transport == "peer" else 0
            ch.ra = self._route_args(ch)
            if self.global_batch:
                # phase 1, then every rank's totals; slot_base = sum over the lower ranks
                check(lib.moe_stage_route_counts(ctypes.byref(ch.ra), ctypes.byref(ch.dims),
                                                 self.raw.data_ptr(), sp))
                allraw = torch.empty(self.world, *self.raw.shape, dtype=torch.int32, device=self.device)
                dist.all_gather_into_tensor(allraw, self.raw, group=self.group)
                torch.sum(allraw[: self.rank], dim=0, dtype=torch.int32, out=self.slot_base)
                ch.dims.slot_base = self.slot_base.data_ptr()
                check(lib.moe_stage_route_finish(ctypes.byref(ch.ra), ctypes.byref(ch.dims), sp))
            else:
                check(lib.moe_stage_route(ctypes.byref(ch.ra), ctypes.byref(ch.dims), sp))
        ev("routed")
        if self.transport == "peer":
            ch = self.chunks[0]
            ch.ra.hidden_mlp_layer_2_out = self.peer_local["back_y"]   # combine reads the peer-written rows
            self._forward_peer(S, ev)
            ev("combine")
            check(lib.moe_stage_combine(ctypes.byref(ch.ra), ctypes.byref(ch.dims), sp))
            ev("end")
            return self.out
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
        with torch.cuda.stream(C):                          # 3. rows (and row scales) to owners
            C.wait_event(routed)
            for ch, (ss, rs, _) in zip(self.chunks, plans):
                works = [dist.all_to_all_single(ch.recv_x[:sum(rs)], ch.send_x[:sum(ss)], rs, ss,
                                                group=self.group, async_op=True)]
                if self.n_scale:
                    works.append(dist.all_to_all_single(ch.recv_scale[:sum(rs)], ch.send_scale[:sum(ss)], rs, ss,
                                                        group=self.group, async_op=True))
                sends.append(works)
        rets = []
        fdims = self._ffn_dims_base()
        for ch, (ss, rs, (g_rows, g_start, g_exp)), works in zip(self.chunks, plans, sends):
            for work in works:
                work.wait()                                  # compute stream waits for chunk's rows
            ev("ffn")
            fa = self._ffn_args(ch)
            fd = MoeDims(*[getattr(fdims, n) for n, _ in MoeDims._fields_])
            fd.scratch, fd.scratch_bytes = ch.ffn_scratch.data_ptr(), ch.ffn_scratch.numel()
            if self.n_scale:
                fd.act_scale = ch.recv_scale.data_ptr()
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
