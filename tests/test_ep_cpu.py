"""Expert-parallel host logic on CPU: the planner (pure functions of
sparsemoe_b200.ep) and the full exchange pattern over a world-size-2 gloo
group, with the oracle's routing and an f32 host FFN standing in for the GPU
stages.  The exchanged result must equal the single-process layer."""
import os

import numpy as np
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import sparsemoe_b200 as sm
from sparsemoe_b200.ep import recv_plan, send_splits
from oracle import oracle as O


def test_send_splits_and_recv_plan():
    table = np.array([[3, 0, 5, 1], [2, 4, 0, 6]], np.int32)      # P=2 senders, E=4
    assert send_splits(table[0], 2) == [3, 6]
    assert send_splits(table[1], 2) == [6, 6]
    rsplit, (rows, start, exp) = recv_plan(table, 0)              # owner 0: experts 0, 1
    assert rsplit == [3, 6]
    # groups ordered (local expert, sender); receive buffer = [s0: e0 e1][s1: e0 e1]
    assert rows.tolist() == [3, 2, 0, 4]
    assert start.tolist() == [0, 3, 3, 5]
    assert exp.tolist() == [0, 0, 1, 1]
    rsplit, (rows, start, exp) = recv_plan(table, 1)              # owner 1: experts 2, 3
    assert rsplit == [6, 6] and rows.tolist() == [5, 0, 1, 6] and start.tolist() == [0, 6, 5, 6]


def _to_f32(u16):
    return u16.view(np.float16).astype(np.float32)


def _dense_rows(r, cfg, cap):
    """The dense expert-major row order of moe_stage_route: for each expert e,
    batches in order, slots in order -> (token index, route index)."""
    B, N, E, k = cfg.num_batches, cfg.tokens, cfg.num_experts, cfg.top_k
    order = []
    for e in range(E):
        for b in range(B):
            for s in range(int(r["counts"][b, e])):
                t = int(r["token_ids"][b, e, s])
                order.append(b * N + t)
    return order


def _ffn_rows(a16, wg, wu, wd):
    a = _to_f32(a16)
    g = a @ _to_f32(wg)
    u = a @ _to_f32(wu)
    h = (u * (g / (1 + np.exp(-g)))).astype(np.float16).astype(np.float32)
    return (h @ _to_f32(wd)).astype(np.float32)


def _rank_main(rank, world, port, cfg_args, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    cfg = sm.LayerConfig(*cfg_args)
    full = sm.make_inputs(cfg, 5)                      # same weights everywhere
    mine = sm.make_inputs(cfg, 100 + rank)             # this rank's own tokens
    cap = cfg.capacity()
    r = O.route(mine["x"], full["wr"], None, cfg.num_batches, cfg.tokens, cfg.d_model, cfg.num_experts,
                cfg.top_k, cap, False)
    order = _dense_rows(r, cfg, cap)
    send_x = mine["x"][order] if order else np.zeros((0, cfg.d_model), np.uint16)
    rows_e = r["counts"].sum(axis=0).astype(np.int32)
    table = [torch.zeros(cfg.num_experts, dtype=torch.int32) for _ in range(world)]
    dist.all_gather(table, torch.from_numpy(rows_e))
    table = torch.stack(table).numpy()
    ss = send_splits(table[rank], world)
    rs, (g_rows, g_start, g_exp) = recv_plan(table, rank)
    # 16-bit rows travel as int32 pairs (gloo has no 16-bit all-to-all)
    recv = torch.empty(sum(rs), cfg.d_model // 2, dtype=torch.int32)
    dist.all_to_all_single(recv, torch.from_numpy(np.ascontiguousarray(send_x).view(np.int32)), rs, ss)
    recv = recv.numpy().view(np.uint16)
    e_loc = cfg.num_experts // world
    y = np.zeros((recv.shape[0], cfg.d_model), np.float32)
    for n, st, j in zip(g_rows, g_start, g_exp):
        e = rank * e_loc + j
        if n:
            y[st:st + n] = _ffn_rows(recv[st:st + n], full["wg"][e], full["wu"][e], full["wd"][e])
    back = torch.empty(sum(ss), cfg.d_model, dtype=torch.float32)
    dist.all_to_all_single(back, torch.from_numpy(y), ss, rs)
    back = back.numpy()
    # combine: route -> its row in the dense layout
    start = np.concatenate([[0], np.cumsum(rows_e)])
    rowbase = np.zeros((cfg.num_batches, cfg.num_experts), np.int64)
    for e in range(cfg.num_experts):
        acc = 0
        for b in range(cfg.num_batches):
            rowbase[b, e] = acc
            acc += r["counts"][b, e]
    out = np.zeros((cfg.T, cfg.d_model), np.float32)
    for t in range(cfg.T):
        b = t // cfg.tokens
        for l in range(cfg.top_k):
            ri = t * cfg.top_k + l
            if r["route_slot"][ri] >= 0:
                e = r["idx"][t, l]
                out[t] += r["w"][t, l] * back[start[e] + rowbase[b, e] + r["route_slot"][ri]]
    ref = O.forward({**full, "x": mine["x"]}, cfg)["out"]
    results[rank] = float(np.abs(out - ref).max() / np.abs(ref).max())
    dist.destroy_process_group()


def test_ep_exchange_gloo_world2():
    cfg_args = (2, 96, 256, 128, 8, 2, 1.0)
    port = 29500 + (os.getpid() % 2000)
    with mp.Manager() as m:
        results = m.dict()
        mp.spawn(_rank_main, args=(2, port, cfg_args, results), nprocs=2, join=True)
        errs = dict(results)
    assert set(errs) == {0, 1}
    assert max(errs.values()) < 1e-2, errs


def _global_rank_main(rank, world, port, cfg_args, results):
    """A batch of world*N tokens split over the ranks: each rank routes its
    shard, the per-expert totals are all-gathered and a route is kept iff
    (sum of the lower ranks' totals) + its slot within the shard < CAP of the
    whole batch.  Must equal the single-process routing of the whole batch."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    B, N, d, f, E, k, cf, zipf = cfg_args
    full_cfg = sm.LayerConfig(B, N * world, d, f, E, k, cf, zipf_s=zipf)
    full = sm.make_inputs(full_cfg, 3)
    cap = full_cfg.capacity()
    ref = O.route(full["x"], full["wr"], full["bias"], B, N * world, d, E, k, cap, False)
    x = full["x"].reshape(B, world, N, d)[:, rank].reshape(B * N, d)
    # local routing with no drop (cap = N) gives the shard's route-order slots
    loc = O.route(x, full["wr"], full["bias"], B, N, d, E, k, N * k, False)
    raw = np.zeros((B, E), np.int32)
    for b in range(B):
        raw[b] = np.bincount(loc["idx"][b * N:(b + 1) * N].reshape(-1), minlength=E)[:E]
    gathered = [torch.zeros(B, E, dtype=torch.int32) for _ in range(world)]
    dist.all_gather(gathered, torch.from_numpy(raw))
    slot_base = sum(g.numpy() for g in gathered[:rank]) if rank else np.zeros((B, E), np.int32)
    ok = True
    for b in range(B):
        for t in range(N):
            for l in range(k):
                r = (b * N + t) * k + l
                e = loc["idx"][b * N + t, l]
                kept = loc["route_slot"][r] >= 0 and slot_base[b, e] + loc["route_slot"][r] < cap
                gr = (b * N * world + rank * N + t) * k + l
                ok &= bool(ref["idx"][b * N * world + rank * N + t, l] == e)
                ok &= bool(kept == (ref["route_slot"][gr] >= 0))
                if kept:
                    ok &= bool(slot_base[b, e] + loc["route_slot"][r] == ref["route_slot"][gr])
    results[rank] = ok
    dist.destroy_process_group()


def test_global_batch_drops_gloo_world2():
    cfg_args = (2, 96, 256, 128, 16, 4, 1.0, 1.2)       # Zipf bias: hot experts overflow CAP
    port = 29700 + (os.getpid() % 2000)
    with mp.Manager() as m:
        results = m.dict()
        mp.spawn(_global_rank_main, args=(2, port, cfg_args, results), nprocs=2, join=True)
        res = dict(results)
    assert res == {0: True, 1: True}


def test_ep_plan_host_matches_recv_plan():
    """The peer transport's plan (host restatement of moe_ep_plan) agrees with
    the NCCL transport's planner for contiguous ownership: same owner-side
    groups, and each sender's rows land after the blocks of lower senders."""
    from sparsemoe_b200.ep import ep_plan_host
    rng = np.random.default_rng(0)
    P, E = 4, 16
    table = rng.integers(0, 50, (P, E)).astype(np.int32)
    for rank in range(P):
        plan = ep_plan_host(table, rank)
        _, (rows, start, exp) = recv_plan(table, rank)
        assert np.array_equal(plan[2 * E:3 * E], rows)
        assert np.array_equal(plan[3 * E:4 * E], start)
        assert np.array_equal(plan[4 * E:5 * E], exp)
        # group (j, s) results go to expert rank*E/P + j's first row in sender s's dense layout
        el = E // P
        for g in range(E):
            j, s = divmod(g, P)
            assert plan[6 * E + g] == table[s, :rank * el + j].sum()
    # strided ownership: every expert has exactly one owner and each owner's groups cover its experts
    for rank in range(P):
        plan = ep_plan_host(table, rank, strided=True)
        assert np.array_equal(plan[:E], np.arange(E) % P)
        assert np.array_equal(plan[2 * E:3 * E].reshape(E // P, P), table[:, rank::P].T)


def _peer_rank_main(rank, world, port, strided, results):
    """The peer transport's data movement on CPU: each rank routes its shard of
    one global batch (global CAP via the slot_base prefix), places its kept
    rows with the device plan's host restatement (ep_plan_host), the owners
    run the FFN over the plan's row groups and send each result row to the
    row the plan names in the sender's layout, and the sender combines.  Must
    equal the single-process layer on the whole batch, for contiguous and
    strided expert ownership."""
    from sparsemoe_b200.ep import ep_plan_host
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    N, d, f, E, k = 48, 256, 128, 8, 2
    full_cfg = sm.LayerConfig(1, N * world, d, f, E, k, 1.0, zipf_s=1.0)
    full = sm.make_inputs(full_cfg, 9)
    cap = full_cfg.capacity()
    ref = O.forward(full, full_cfg, nthreads=2)
    x = full["x"][rank * N:(rank + 1) * N]
    loc = O.route(x, full["wr"], full["bias"], 1, N, d, E, k, N * k, False)      # shard slots, no drop yet
    raw = np.bincount(loc["idx"].reshape(-1), minlength=E).astype(np.int32)
    every = [torch.zeros(E, dtype=torch.int32) for _ in range(world)]
    dist.all_gather(every, torch.from_numpy(raw))
    base = sum(t.numpy() for t in every[:rank]) if rank else np.zeros(E, np.int32)
    # kept routes of this shard, dense expert-major (expert, slot) order
    kept = {}
    for r in range(N * k):
        e, s = loc["idx"].reshape(-1)[r], loc["route_slot"][r]
        if s >= 0 and base[e] + s < cap:
            kept.setdefault(e, []).append((s, r))
    table_mine = np.array([len(kept.get(e, [])) for e in range(E)], np.int32)
    every = [torch.zeros(E, dtype=torch.int32) for _ in range(world)]
    dist.all_gather(every, torch.from_numpy(table_mine))
    table = np.stack([t.numpy() for t in every])
    plan = ep_plan_host(table, rank, strided)
    start = np.concatenate([[0], np.cumsum(table_mine)])          # my dense layout
    # dispatch: (owner, receive row, token row) for every kept route of mine
    msgs = []
    for e, lst in kept.items():
        for i, (_, r) in enumerate(sorted(lst)):
            msgs.append((int(plan[e]), int(plan[E + e]) + i, r // k))
    got = [None] * world
    dist.all_gather_object(got, [(q, row, x[t].tolist()) for q, row, t in msgs])
    recv = {}
    for lst in got:
        for q, row, vals in lst:
            if q == rank:
                recv[row] = np.array(vals, np.uint16)
    # owner FFN over the plan's groups; results to (sender, row in its layout)
    outs = []
    P = world
    for g in range(E):
        n, st, j, snd, orow = (int(plan[c * E + g]) for c in range(2, 7))
        ge = j * P + rank if strided else rank * (E // P) + j
        for i in range(n):
            y = _ffn_rows(recv[st + i][None, :], full["wg"][ge], full["wu"][ge], full["wd"][ge])[0]
            outs.append((snd, orow + i, y.tolist()))
    got = [None] * world
    dist.all_gather_object(got, outs)
    back = np.zeros((int(start[-1]), d), np.float32)
    for lst in got:
        for snd, row, vals in lst:
            if snd == rank:
                back[row] = vals
    # combine in route order
    out = np.zeros((N, d), np.float32)
    for t in range(N):
        for l in range(k):
            r = t * k + l
            e = loc["idx"][t, l]
            lst = sorted(kept.get(e, []))
            pos = [rr for _, rr in lst]
            if r in pos:
                out[t] += loc["w"][t, l] * back[start[e] + pos.index(r)]
    err = float(np.abs(out - ref["out"][rank * N:(rank + 1) * N]).max() / np.abs(ref["out"]).max())
    results[rank] = err
    dist.destroy_process_group()


def test_peer_transport_plan_gloo_world2():
    for strided in (False, True):
        port = 29900 + (os.getpid() % 1000) + (7 if strided else 0)
        with mp.Manager() as m:
            results = m.dict()
            mp.spawn(_peer_rank_main, args=(2, port, strided, results), nprocs=2, join=True)
            errs = dict(results)
        assert set(errs) == {0, 1}
        assert max(errs.values()) < 1e-2, (strided, errs)


def _simulate_ranks(P, strided, B=2, N=32, d=256, E=32, k=4, cf=1.0, zipf=1.2, seed=11):
    """P expert-parallel ranks in one process, at the level of row indices:
    each rank routes its shard of every global batch, the global drop rule
    keeps a route iff (lower ranks' totals) + its shard slot < CAP, every kept
    row is placed with the sender's plan and found again through the owner's
    plan, and the owner's result row goes back to the sender's dense slot."""
    from sparsemoe_b200.ep import ep_plan_host
    full_cfg = sm.LayerConfig(B, N * P, d, 128, E, k, cf, zipf_s=zipf)
    full = sm.make_inputs(full_cfg, seed)
    cap = full_cfg.capacity()
    ref = O.route(full["x"], full["wr"], full["bias"], B, N * P, d, E, k, cap, False)
    xs = full["x"].reshape(B, P, N, d)
    loc = [O.route(np.ascontiguousarray(xs[:, q]).reshape(B * N, d), full["wr"], full["bias"],
                   B, N, d, E, k, N * k, False) for q in range(P)]
    raw = np.zeros((P, B, E), np.int64)
    for q in range(P):
        for b in range(B):
            raw[q, b] = np.bincount(loc[q]["idx"][b * N:(b + 1) * N].reshape(-1), minlength=E)[:E]
    # (1) global drops, bit-exact against the single-rank routing of the whole batch
    kept = [dict() for _ in range(P)]          # kept[q][(b, e)] = route ids in slot order
    for q in range(P):
        base = raw[:q].sum(axis=0)
        idx, slot = loc[q]["idx"], loc[q]["route_slot"]
        for b in range(B):
            for t in range(N):
                for l in range(k):
                    r = (b * N + t) * k + l
                    gt = b * N * P + q * N + t
                    e = int(idx[b * N + t, l])
                    assert e == ref["idx"][gt, l]
                    keep = slot[r] >= 0 and base[b, e] + slot[r] < cap
                    assert keep == (ref["route_slot"][gt * k + l] >= 0)
                    if keep:
                        assert base[b, e] + slot[r] == ref["route_slot"][gt * k + l]
                        kept[q].setdefault((b, e), []).append((int(slot[r]), r))
    for q in range(P):
        for key in kept[q]:
            kept[q][key].sort()
    # each sender's dense layout: expert-major, then batch, then slot
    dense = []
    for q in range(P):
        order = [(e, r) for e in range(E) for b in range(B) for _, r in kept[q].get((b, e), [])]
        dense.append(order)
    table = np.array([[sum(1 for ee, _ in dense[q] if ee == e) for e in range(E)] for q in range(P)], np.int32)
    plans = [ep_plan_host(table, q, strided).astype(np.int64) for q in range(P)]
    # (2) dispatch: (owner, receive row) of every kept row, unique and dense per owner
    where = {}
    for q in range(P):
        seen = {}
        for pos, (e, r) in enumerate(dense[q]):
            i = seen.get(e, 0)
            seen[e] = i + 1
            dst = (int(plans[q][e]), int(plans[q][E + e]) + i)
            assert dst not in where
            where[dst] = (q, e, pos)
    for o in range(P):
        rows = sorted(row for (own, row) in where if own == o)
        assert rows == list(range(len(rows)))
    # (3) the owner's groups find every row and send its result to the sender's dense slot
    back = set()
    el = E // P
    for o in range(P):
        pl = plans[o]
        for g in range(E):
            n, st, j, snd, orow = (int(pl[c * E + g]) for c in range(2, 7))
            ge = j * P + o if strided else o * el + j
            assert (ge % P == o) if strided else (ge // el == o)
            for i in range(n):
                q, e, pos = where[(o, st + i)]
                assert (q, e) == (snd, ge)
                assert orow + i == pos
                back.add((q, pos))
    assert back == {(q, pos) for q in range(P) for pos in range(len(dense[q]))}
    return int(table.sum()), int(ref["counts"].sum())


def test_ep_simulated_ranks_up_to_8():
    """Partition, global drops and the peer plan as 2, 4 and 8 ranks in one
    process, for contiguous and strided expert ownership: the kept set and
    slots equal the single-rank routing bit for bit and every kept row makes
    the round trip sender -> owner -> sender to its own slot."""
    for P in (2, 4, 8):
        for strided in (False, True):
            kept_rows, ref_rows = _simulate_ranks(P, strided)
            assert kept_rows == ref_rows and kept_rows < 2 * 32 * P * 4     # Zipf bias: drops happen
            kept_rows, ref_rows = _simulate_ranks(P, strided, cf=2.0, zipf=0.0)
            assert kept_rows == ref_rows
