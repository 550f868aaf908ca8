"""CPU oracle checks (no GPU): golden vectors from the reference's own GPU
code, the reference's known answer, and an independent numpy restatement of
the routing stages on small cases."""
import numpy as np
import pytest

import sparsemoe_b200 as sm
from oracle import oracle as O
from oracle.make_golden import layer_config


@pytest.mark.parametrize("name", ["k2", "k4"])
def test_oracle_matches_reference_gpu_golden(name):
    """tests/golden/ref_unfused_*.npz: the reference's kernels/unfused.cu run on
    a B200 (oracle/make_golden.py).  Same seeded inputs, no capacity drop."""
    from pathlib import Path
    g = np.load(Path(__file__).parent / "golden" / f"ref_unfused_{name}.npz")
    cfg, seed, _ = layer_config(name)
    r = O.forward(sm.make_inputs(cfg, seed), cfg)
    # logits: WMMA order vs the fixed order -> equal to f32 rounding
    np.testing.assert_allclose(r["logits"], g["logits"], rtol=0, atol=1e-5)
    assert np.array_equal(r["idx"], g["idx"])
    np.testing.assert_allclose(r["w"], g["w"], rtol=0, atol=2e-6)
    assert np.array_equal(r["counts"], g["counts"])
    out = r["out"][g["out_rows"]]
    err = np.abs(out - g["out"]).max() / np.abs(g["out"]).max()
    assert err < 1e-3, err


def test_known_answer_zero_inputs():
    """The reference's only workload: all-zero x and router (inputs/data.cu:164-177,
    237-243) -> experts 0..k-1, weights 1/k, counts min(N, CAP) for e < k, zero output."""
    cfg = sm.LayerConfig(4, 256, 256, 256, 32, 4, 0.8)
    z = {k: (None if v is None else np.zeros_like(v)) for k, v in sm.make_inputs(cfg, 0).items()}
    r = O.forward(z, cfg)
    assert (r["idx"] == np.arange(4)).all()
    assert np.allclose(r["w"], 0.25)
    cap = cfg.capacity()
    assert cap == 32
    exp = np.zeros((4, 32), np.int32)
    exp[:, :4] = min(256, cap)
    assert np.array_equal(r["counts"], exp)
    assert not np.any(r["out"])


def numpy_route(logits, k, cap, B, N, E):
    """Independent restatement of capacity.cu:171-309 on given logits."""
    T = B * N
    idx = np.full((T, k), -1, np.int64)
    for t in range(T):
        cand = [(-float(v), e) for e, v in enumerate(logits[t]) if v > -1e20]   # NaN fails '>'
        cand.sort()
        for l, (_, e) in enumerate(cand[:k]):
            idx[t, l] = e
    slots = np.full(T * k, -1, np.int64)
    counts = np.zeros((B, E), np.int64)
    for b in range(B):
        c = np.zeros(E, np.int64)
        for r in range(N * k):
            e = idx.reshape(-1)[b * N * k + r]
            if e < 0:
                continue
            if c[e] < cap:
                slots[b * N * k + r] = c[e]
            c[e] += 1
        counts[b] = np.minimum(c, cap)
    return idx, slots, counts


@pytest.mark.parametrize("seed,zipf", [(0, 0.0), (1, 1.1), (2, 2.0)])
def test_routing_matches_numpy_restatement(seed, zipf):
    cfg = sm.LayerConfig(2, 96, 256, 128, 16, 3, 0.9, zipf_s=zipf)
    inp = sm.make_inputs(cfg, seed)
    cap = cfg.capacity()
    r = O.route(inp["x"], inp["wr"], inp["bias"], 2, 96, 256, 16, 3, cap, False)
    idx, slots, counts = numpy_route(r["logits"], 3, cap, 2, 96, 16)
    assert np.array_equal(r["idx"], idx)
    assert np.array_equal(r["route_slot"], slots)
    assert np.array_equal(r["counts"], counts)
    if zipf >= 2.0:
        assert (slots < 0).any()


def test_logit_order_matches_python_restatement():
    """The fixed f32 order: 32 lane partials over interleaved 8-element chunks
    (fmaf chains), xor butterfly, then + bias."""
    cfg = sm.LayerConfig(1, 5, 512, 128, 8, 2, 1.0, zipf_s=1.0)
    inp = sm.make_inputs(cfg, 4)
    r = O.route(inp["x"], inp["wr"], inp["bias"], 1, 5, 512, 8, 2, 16, False)
    x = inp["x"].view(np.float16).astype(np.float64)
    w = inp["wr"].view(np.float16).astype(np.float64)
    for t in range(5):
        for e in range(8):
            p = []
            for lane in range(32):
                acc = np.float32(0)
                for c in range(lane, 512 // 8, 32):
                    for j in range(8 * c, 8 * c + 8):
                        # fmaf: exact product (16-bit inputs) + one rounding
                        acc = np.float32(np.float64(acc) + x[t, j] * w[j, e])
                p.append(acc)
            for off in (16, 8, 4, 2, 1):
                p = [np.float32(p[i] + p[i ^ off]) for i in range(32)]
            v = np.float32(p[0] + inp["bias"][e])
            assert v == r["logits"][t, e]


def test_nan_and_tie_semantics():
    """NaN logits are never selected (sentinel -1e20 / -1 remain, capacity.cu:200-212);
    equal logits go to the lower expert index."""
    cfg = sm.LayerConfig(1, 4, 256, 128, 8, 2, 2.0)
    inp = sm.make_inputs(cfg, 0)
    x = inp["x"].copy()
    x[1, 0] = 0x7E00                    # f16 NaN -> every logit of token 1 is NaN
    wr = inp["wr"].copy()
    wr[:, 6] = wr[:, 3]                 # experts 3 and 6 tie for every token
    r = O.route(x, wr, None, 1, 4, 256, 8, 2, 16, False)
    assert (r["idx"][1] == -1).all()
    np.testing.assert_allclose(r["w"][1], 0.5)
    for t in (0, 2, 3):
        if 6 in r["idx"][t]:
            assert 3 in r["idx"][t] and list(r["idx"][t]).index(3) < list(r["idx"][t]).index(6)


def test_e4m3_encoder_matches_product_quantiser():
    """The oracle's e4m3 rounding (restated from the format) agrees with the
    library's block quantiser on random blocks, including saturation at 448
    and subnormals."""
    rng = np.random.default_rng(1)
    w = (rng.standard_normal((2, 256, 128)) * np.array([1e-4, 1.0])[:, None, None]).astype(np.float32)
    w[0, 0, 0] = 0.0
    w[1, 5, 7] = -3.0e4
    b16 = (w.view(np.uint32) >> 16).astype(np.uint16)       # truncate to bf16 bit patterns
    q, sc = sm.quantize_fp8_blocks(b16, bf16=True)
    vals = (b16.astype(np.uint32) << 16).view(np.float32)
    L = O.lib()
    for e in range(2):
        for kb in range(2):
            blk = vals[e, kb * 128:(kb + 1) * 128, :] / sc[e, kb, 0]
            enc = np.array([L.oracle_e4m3(float(v)) for v in blk.reshape(-1)], np.uint8)
            assert np.array_equal(enc, q[e, kb * 128:(kb + 1) * 128, :].reshape(-1))
    assert L.oracle_e4m3(1000.0) == 0x7E and L.oracle_e4m3(-1000.0) == 0xFE
    assert L.oracle_e4m3_decode(0x7E) == 448.0 and L.oracle_e4m3_decode(0x01) == 2.0 ** -9


def _block_tree(b, a, n):
    if n == 1:
        return b[a]
    h = 1
    while 2 * h < n:
        h *= 2
    return np.float32(_block_tree(b, a, h) + _block_tree(b, a + h, n - h))


@pytest.mark.parametrize("d", [256, 1536, 3584])
def test_logit_order_many_experts_is_blocked_tree(d):
    """E >= 64: per (token, expert) one fmaf chain per 512-j block from 0.0f,
    the blocks summed by the tree tree(a, n) = tree(a, h) + tree(a + h, n - h)
    (h the largest power of two below n), then + bias."""
    cfg = sm.LayerConfig(1, 2, d, 128, 64, 2, 1.0, zipf_s=1.0)
    inp = sm.make_inputs(cfg, 2)
    r = O.route(inp["x"], inp["wr"], inp["bias"], 1, 2, d, 64, 2, 16, False)
    x = inp["x"].view(np.float16).astype(np.float64)
    w = inp["wr"].view(np.float16).astype(np.float64)
    nb = (d + 511) // 512
    for t in range(2):
        for e in (0, 17, 63):
            blocks = []
            for b in range(nb):
                acc = np.float32(0)
                for j in range(512 * b, min(d, 512 * b + 512)):
                    acc = np.float32(np.float64(acc) + x[t, j] * w[j, e])   # exact product + one rounding
                blocks.append(acc)
            assert np.float32(_block_tree(blocks, 0, nb) + inp["bias"][e]) == r["logits"][t, e]


def test_int8_channel_quantiser_matches_numpy():
    """Per-output-channel int8: s = amax over K / 127 (1 for a zero column),
    q = clamp(rint(w / s), +-127)."""
    rng = np.random.default_rng(3)
    w = rng.standard_normal((2, 64, 48)).astype(np.float32)
    w[1, :, 5] = 0.0
    b16 = (w.view(np.uint32) >> 16).astype(np.uint16)
    q, sc = sm.quantize_int8_channel(b16, bf16=True)
    vals = (b16.astype(np.uint32) << 16).view(np.float32)
    amax = np.abs(vals).max(axis=1)
    s = np.where(amax > 0, amax / np.float32(127.0), np.float32(1.0)).astype(np.float32)
    assert np.array_equal(sc, s)
    assert np.array_equal(q, np.clip(np.rint(vals / s[:, None, :]), -127, 127).astype(np.int8))


def test_int8_channel_oracle_matches_numpy_restatement():
    """The C oracle's INT8_CHANNEL FFN against an independent numpy restatement
    (exact integer sums, the same f32 scale products, per-block h scales)."""
    cfg = sm.LayerConfig(1, 24, 256, 256, 8, 2, 2.0, dtype=sm.DTYPE_INT8_CHANNEL)
    inp = sm.make_inputs(cfg, 5)
    ref = O.forward(inp, cfg, nthreads=2)
    f32 = np.float32
    x = (inp["x"].astype(np.uint32) << 16).view(np.float32)
    out = np.zeros((cfg.T, cfg.d_model), np.float32)
    for t in range(cfg.T):
        for l in range(cfg.top_k):
            if ref["route_slot"][t * cfg.top_k + l] < 0:
                continue
            e = ref["idx"][t, l]
            amax = np.abs(x[t]).max()
            sx = amax / f32(127) if amax > 0 else f32(1)
            qa = np.clip(np.rint(x[t] / sx), -127, 127).astype(np.int64)
            G = qa @ inp["wg_q"][e].astype(np.int64)
            U = qa @ inp["wu_q"][e].astype(np.int64)
            g = G.astype(np.float32) * (sx * inp["sg"][e])
            u = U.astype(np.float32) * (sx * inp["su"][e])
            h = u * (g / (f32(1) + np.exp(-g)))
            hb = h.reshape(-1, 128)
            hm = np.abs(hb).max(axis=1)
            sh = np.where(hm > 0, hm / f32(127), f32(1)).astype(np.float32)
            qh = np.clip(np.rint(hb / sh[:, None]), -127, 127).astype(np.int64)
            acc = np.zeros(cfg.d_model, np.float32)
            for kb in range(qh.shape[0]):
                P = qh[kb] @ inp["wd_q"][e, kb * 128:(kb + 1) * 128].astype(np.int64)
                acc = (P.astype(np.float64) * np.float64(sh[kb]) + acc).astype(np.float32)
            y = acc * inp["sd"][e]
            out[t] += ref["w"][t, l] * y
    np.testing.assert_allclose(ref["out"], out, rtol=1e-4, atol=1e-5 * float(np.abs(out).max()))


def test_nvfp4_quantiser_matches_numpy():
    """NVFP4: g = amax/(448*6); per 16 K-rows and column s = e4m3(amax/(6g));
    q = nearest e2m1 (ties to the even code) of w / (s g), saturating at 6."""
    rng = np.random.default_rng(4)
    w = (rng.standard_normal((2, 64, 16)) * 0.1).astype(np.float32)
    w[0, 16:32, 3] = 0.0
    b16 = (w.view(np.uint32) >> 16).astype(np.uint16)
    q, s, g = sm.quantize_nvfp4(b16, bf16=True)
    vals = (b16.astype(np.uint32) << 16).view(np.float32)
    L = O.lib()
    mags = np.array([0, 0.5, 1, 1.5, 2, 3, 4, 6], np.float64)
    for e in range(2):
        ge = np.float32(np.abs(vals[e]).max() / np.float32(448.0 * 6.0))
        assert g[e] == ge
        for grp in range(4):
            blk = vals[e, grp * 16:(grp + 1) * 16]
            for n in range(16):
                m = np.abs(blk[:, n]).max()
                sc = s[e, grp, n]
                if m == 0:
                    assert sc == 0x38
                else:
                    assert sc == L.oracle_e4m3(float(np.float32(m / (np.float32(6.0) * ge))))
                div = np.float32(np.float32(L.oracle_e4m3_decode(int(sc))) * ge)
                for i in range(16):
                    k = grp * 16 + i
                    byte = q[e, k, (n >> 3) * 4 + ((4 * ((n & 7) >> 1) + 16 * (n & 1)) >> 3)]
                    code = (byte >> ((4 * ((n & 7) >> 1) + 16 * (n & 1)) & 7)) & 15
                    a = abs(float(np.float32(blk[i, n] / div)))
                    d = np.abs(mags - a)
                    best = 7 if a >= 6 else min((c for c in range(8) if d[c] == d.min()), key=lambda c: c & 1)
                    assert code & 7 == best, (e, k, n, a, code)
                    if blk[i, n] < 0:
                        assert code & 8


# ---- numpy restatements of the oracle's FFN for the quantised formats -----------
def _bf16_to_f32(u16):
    return (np.asarray(u16, np.uint16).astype(np.uint32) << 16).view(np.float32)


def _round_bf16(v):
    """f32 -> nearest-even bf16 -> f32."""
    u = np.asarray(v, np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return (u.astype(np.uint32) << 16).view(np.float32)


def _nibbles(packed, N):
    """[E, K, N/2] pair-interleaved 4-bit words -> [E, K, N] codes."""
    n = np.arange(N)
    bit = 4 * ((n & 7) >> 1) + 16 * (n & 1)
    byte = (n >> 3) * 4 + (bit >> 3)
    return (packed[:, :, byte] >> (bit & 7)) & 15


def _np_ffn(x, wg, wu, wd, r, k, round_h, T):
    """Route-by-route f32 FFN of dequantised weights (h rounded by round_h),
    combined in route order."""
    out = np.zeros((T, x.shape[1]), np.float32)
    for t in range(T):
        for l in range(k):
            if r["route_slot"][t * k + l] < 0:
                continue
            e = r["idx"][t, l]
            g = (x[t].astype(np.float64) @ wg[e].astype(np.float64)).astype(np.float32)
            u = (x[t].astype(np.float64) @ wu[e].astype(np.float64)).astype(np.float32)
            h = round_h(u * (g / (np.float32(1) + np.exp(-g))))
            y = (h.astype(np.float64) @ wd[e].astype(np.float64)).astype(np.float32)
            out[t] = out[t] + np.float32(r["w"][t, l]) * y
    return out


def _check_close(ref_out, np_out):
    np.testing.assert_allclose(ref_out, np_out, rtol=2e-3, atol=2e-3 * float(np.abs(np_out).max()))


def test_int4_g128_quantiser_matches_numpy():
    rng = np.random.default_rng(6)
    w = (rng.standard_normal((2, 256, 16)) * 0.05).astype(np.float32)
    w[1, :128, 3] = 0.25                               # a constant group: s = 1 (fp16), z = -min
    b16 = (w.view(np.uint32) >> 16).astype(np.uint16)
    q, s, z = sm.quantize_int4_g128(b16, bf16=True)
    vals = _bf16_to_f32(b16)
    codes = _nibbles(q, 16)
    for e in range(2):
        for g in range(2):
            blk = vals[e, g * 128:(g + 1) * 128]
            mn, mx = blk.min(axis=0), blk.max(axis=0)
            sc = ((mx - mn) / np.float32(15)).astype(np.float32)
            sc = np.where(sc > 0, sc, np.float32(1)).astype(np.float32)
            sh = sc.astype(np.float16)
            zh = (-mn / sh.astype(np.float32)).astype(np.float16)
            assert np.array_equal(s[e, g], sh.view(np.uint16)) and np.array_equal(z[e, g], zh.view(np.uint16))
            qq = np.clip(np.rint(blk / sh.astype(np.float32) + zh.astype(np.float32)), 0, 15)
            assert np.array_equal(codes[e, g * 128:(g + 1) * 128], qq)


def test_w4_oracle_matches_numpy_restatement():
    cfg = sm.LayerConfig(1, 16, 256, 256, 8, 2, 1.0, dtype=sm.DTYPE_W4A16, cap=-1)
    inp = sm.make_inputs(cfg, 2)
    ref = O.forward(inp, cfg, nthreads=2)
    x = _bf16_to_f32(inp["x"])

    def deq(n):
        q = _nibbles(inp[n + "_q"], inp[n].shape[2]).astype(np.float64)
        s = inp[n + "_s"].view(np.float16).astype(np.float64).repeat(128, axis=1)
        z = inp[n + "_z"].view(np.float16).astype(np.float64).repeat(128, axis=1)
        return ((q - z) * s).astype(np.float32)
    out = _np_ffn(x, deq("wg"), deq("wu"), deq("wd"), ref, cfg.top_k, _round_bf16, cfg.T)
    _check_close(ref["out"], out)


def test_nvfp4_oracle_matches_numpy_restatement():
    cfg = sm.LayerConfig(1, 16, 256, 256, 8, 2, 1.0, dtype=sm.DTYPE_NVFP4, cap=-1)
    inp = sm.make_inputs(cfg, 2)
    ref = O.forward(inp, cfg, nthreads=2)
    x = _bf16_to_f32(inp["x"])
    L = O.lib()
    e4m3 = np.array([L.oracle_e4m3_decode(i) for i in range(256)], np.float64)
    mag = np.array([0, 0.5, 1, 1.5, 2, 3, 4, 6], np.float64)

    def deq(n):
        c = _nibbles(inp[n + "_q"], inp[n].shape[2])
        v = np.where(c & 8, -1.0, 1.0) * mag[c & 7]
        s = e4m3[inp[n + "_s"]].repeat(16, axis=1)
        return (v * s * inp[n + "_g"].astype(np.float64)[:, None, None]).astype(np.float32)
    out = _np_ffn(x, deq("wg"), deq("wu"), deq("wd"), ref, cfg.top_k, _round_bf16, cfg.T)
    _check_close(ref["out"], out)


def test_fp8_oracle_matches_numpy_restatement():
    """FP8 block path: x and h quantised per 1x128 block (amax/448, e4m3),
    weights e4m3 with 128x128 scales, per-K-block promotion."""
    cfg = sm.LayerConfig(1, 12, 256, 256, 8, 2, 1.0, dtype=sm.DTYPE_FP8_BLOCK, cap=-1)
    inp = sm.make_inputs(cfg, 3)
    ref = O.forward(inp, cfg, nthreads=2)
    L = O.lib()
    dec = np.array([L.oracle_e4m3_decode(i) for i in range(256)], np.float32)

    def q_row(v):
        qv, sc = np.empty_like(v), np.empty(v.size // 128, np.float32)
        for b in range(v.size // 128):
            blk = v[b * 128:(b + 1) * 128]
            m = np.abs(blk).max()
            s = np.float32(m / np.float32(448)) if m > 0 else np.float32(1)
            sc[b] = s
            qv[b * 128:(b + 1) * 128] = dec[[L.oracle_e4m3(float(np.float32(t / s))) for t in blk]]
        return qv, sc
    x = _bf16_to_f32(inp["x"])
    out = np.zeros((cfg.T, cfg.d_model), np.float32)
    for t in range(cfg.T):
        for l in range(cfg.top_k):
            if ref["route_slot"][t * cfg.top_k + l] < 0:
                continue
            e = ref["idx"][t, l]
            qa, sa = q_row(x[t])

            def gemm(qv, sv, wq, ws):
                K, N = wq.shape
                acc = np.zeros(N, np.float32)
                for kb in range(K // 128):
                    p = (qv[kb * 128:(kb + 1) * 128].astype(np.float64) @
                         dec[wq[kb * 128:(kb + 1) * 128]].astype(np.float64)).astype(np.float32)
                    acc = (p.astype(np.float64) * (sv[kb] * ws[kb].repeat(128)).astype(np.float32) + acc).astype(np.float32)
                return acc
            g = gemm(qa, sa, inp["wg_q"][e], inp["sg"][e])
            u = gemm(qa, sa, inp["wu_q"][e], inp["su"][e])
            h = u * (g / (np.float32(1) + np.exp(-g)))
            qh, sh = q_row(h.astype(np.float32))
            y = gemm(qh, sh, inp["wd_q"][e], inp["sd"][e])
            out[t] = out[t] + np.float32(ref["w"][t, l]) * y
    _check_close(ref["out"], out)


def test_int8_per_tensor_oracle_matches_numpy_restatement():
    """The reference's int8 format (capacity_int8_ptx.cu): per-tensor x / h
    quantisation with the MoEArgs scales, exact s32 GEMMs, f32 dequant."""
    cfg = sm.LayerConfig(1, 16, 256, 256, 8, 2, 1.0, dtype=sm.DTYPE_INT8, cap=-1, act_scale=0.03, mid_scale=0.02)
    inp = sm.make_inputs(cfg, 4)
    ref = O.forward(inp, cfg, nthreads=2)
    f32 = np.float32
    x = inp["x"].view(np.float16).astype(np.float32)
    s_in, s_mid = f32(inp["s_in"]), f32(inp["s_mid"])
    out = np.zeros((cfg.T, cfg.d_model), np.float32)
    for t in range(cfg.T):
        for l in range(cfg.top_k):
            if ref["route_slot"][t * cfg.top_k + l] < 0:
                continue
            e = ref["idx"][t, l]
            a = np.rint(np.clip(x[t] / s_in, -128, 127)).astype(np.int64)
            G = a @ inp["wg_q"][e].astype(np.int64)
            U = a @ inp["wu_q"][e].astype(np.int64)
            gf = G.astype(np.float32) * f32(s_in * f32(inp["s_gate"]))
            uf = U.astype(np.float32) * f32(s_in * f32(inp["s_up"]))
            h = np.rint(np.clip(uf * (gf / (f32(1) + np.exp(-gf))) * (f32(1) / s_mid), -128, 127)).astype(np.int64)
            y = (h @ inp["wd_q"][e].astype(np.int64)).astype(np.float32) * f32(s_mid * f32(inp["s_down"]))
            out[t] = out[t] + f32(ref["w"][t, l]) * y
    _check_close(ref["out"], out)


@pytest.mark.parametrize("B,N,E,k,cf,zipf", [(2, 64, 8, 2, 1.0, 1.5), (1, 96, 16, 16, 1.0, 0.0),
                                             (3, 40, 32, 4, 0.5, 1.0), (1, 1, 8, 8, 1.0, 0.0)])
def test_capacity_drop_invariants(B, N, E, k, cf, zipf):
    """Stage 3 (capacity.cu:245-309 in route-id order): per (batch, expert) the
    kept routes are exactly the first CAP routes in route-id order, slots are
    0..count-1 in that order, counts = min(routes, CAP), token_ids / weights
    hold the kept routes' tokens and gate weights, and slots past the count
    stay empty.  Includes k = E (every expert selected) and a single token."""
    cfg = sm.LayerConfig(B, N, 256, 128, E, k, cf, zipf_s=zipf)
    inp = sm.make_inputs(cfg, 4)
    cap = cfg.capacity()
    r = O.route(inp["x"], inp["wr"], inp["bias"], B, N, 256, E, k, cap, False)
    if k == E:
        assert (np.sort(r["idx"], axis=1) == np.arange(E)).all()
    for b in range(B):
        seen = np.zeros(E, np.int64)
        for t in range(N):
            for l in range(k):
                rid = (b * N + t) * k + l
                e = r["idx"][b * N + t, l]
                s = r["route_slot"][rid]
                if seen[e] < cap:
                    assert s == seen[e]
                    assert r["token_ids"][b, e, s] == t
                    assert r["token_weights"][b, e, s] == r["w"][b * N + t, l]
                else:
                    assert s == -1
                seen[e] += 1
        assert np.array_equal(r["counts"][b], np.minimum(seen, cap))
        for e in range(E):
            assert (r["token_ids"][b, e, r["counts"][b, e]:] == -1).all()
            assert (r["token_weights"][b, e, r["counts"][b, e]:] == 0).all()


def test_empty_batch_routes_nothing():
    """T = 0: no routes, zero counts, nothing written."""
    r = O.route(np.zeros((0, 256), np.uint16), np.zeros((256, 8), np.uint16), None, 1, 0, 256, 8, 2, 16, False)
    assert r["idx"].shape == (0, 2) and (r["counts"] == 0).all() and (r["token_ids"] == -1).all()


def _np_per_tensor_ffn(inp, ref, cfg, wq, quant, deq):
    """Route-by-route restatement of the reference's per-tensor paths: a =
    quant(x / s_in), exact / f64 GEMMs, uf = U s_in s_up, gf = G s_in s_gate,
    h = quant(uf * silu(gf) / s_mid), y = Y s_mid s_down, route-order combine."""
    f32 = np.float32
    x = inp["x"].view(np.float16).astype(np.float32)
    s_in, s_mid = f32(inp["s_in"]), f32(inp["s_mid"])
    out = np.zeros((cfg.T, cfg.d_model), np.float32)
    for t in range(cfg.T):
        for l in range(cfg.top_k):
            if ref["route_slot"][t * cfg.top_k + l] < 0:
                continue
            e = ref["idx"][t, l]
            a = deq(quant(x[t] / s_in))
            G = (a @ wq["wg"][e]).astype(np.float32)
            U = (a @ wq["wu"][e]).astype(np.float32)
            gf = G * f32(s_in * f32(inp["s_gate"]))
            uf = U * f32(s_in * f32(inp["s_up"]))
            h = deq(quant(uf * (gf / (f32(1) + np.exp(-gf))) * (f32(1) / s_mid)))
            y = (h @ wq["wd"][e]).astype(np.float32) * f32(s_mid * f32(inp["s_down"]))
            out[t] = out[t] + f32(ref["w"][t, l]) * y
    return out


def test_int4ptx_packing_matches_reference_layout():
    """inputs/data.cu:89-140: byte (n/2, k) of each expert holds column n in
    its low nibble (even n) or high nibble (odd n)."""
    cfg = sm.LayerConfig(1, 4, 256, 128, 8, 2, 1.0, dtype=sm.DTYPE_INT4_PTX)
    inp = sm.make_inputs(cfg, 1)
    q, P = inp["wg_i4"], inp["wg_q"]                   # [E, K, N] values, [E, N/2, K] bytes
    assert P.shape == (8, 64, 256) and q.min() >= -7 and q.max() <= 7
    lo = (P & 15).astype(np.int8)
    hi = (P >> 4).astype(np.int8)
    lo = np.where(lo >= 8, lo - 16, lo)
    hi = np.where(hi >= 8, hi - 16, hi)
    assert np.array_equal(lo.transpose(0, 2, 1), q[:, :, 0::2])
    assert np.array_equal(hi.transpose(0, 2, 1), q[:, :, 1::2])


def test_int4ptx_oracle_matches_numpy_restatement():
    """The reference's int4 format (capacity_int4_ptx.cu): clamps at +-7."""
    cfg = sm.LayerConfig(1, 16, 256, 256, 8, 2, 1.0, dtype=sm.DTYPE_INT4_PTX, cap=-1, act_scale=0.3,
                         mid_scale=0.05)
    inp = sm.make_inputs(cfg, 4)
    ref = O.forward(inp, cfg, nthreads=2)
    wq = {n: inp[n + "_i4"].astype(np.float64) for n in ("wg", "wu", "wd")}
    out = _np_per_tensor_ffn(inp, ref, cfg, wq, lambda v: np.rint(np.clip(v, -7, 7)), lambda q: q.astype(np.float64))
    _check_close(ref["out"], out)
    assert np.abs(out).max() > 0


def test_fp8pt_oracle_matches_numpy_restatement():
    """The reference's fp8 format (capacity_fp8_ptx.cu): e4m3 operands with
    unit weight scales, clamps at +-448."""
    cfg = sm.LayerConfig(1, 12, 256, 256, 8, 2, 1.0, dtype=sm.DTYPE_FP8, cap=-1, act_scale=0.02, mid_scale=0.001)
    inp = sm.make_inputs(cfg, 3)
    ref = O.forward(inp, cfg, nthreads=2)
    L = O.lib()
    dec = np.array([L.oracle_e4m3_decode(i) for i in range(256)], np.float64)
    wq = {n: dec[inp[n + "_q"]] for n in ("wg", "wu", "wd")}

    def quant(v):
        v = np.clip(v, -448, 448)
        return np.array([L.oracle_e4m3(float(t)) for t in v.reshape(-1)], np.uint8).reshape(v.shape)
    out = _np_per_tensor_ffn(inp, ref, cfg, wq, quant, lambda q: dec[q])
    _check_close(ref["out"], out)
    assert np.abs(out).max() > 0


def test_fp8pt_weight_cast_is_the_reference_cast():
    """inputs/data.cu:142-150: e4m3 = nearest-even cast of the fp16 weight."""
    cfg = sm.LayerConfig(1, 4, 256, 128, 8, 2, 1.0, dtype=sm.DTYPE_FP8)
    inp = sm.make_inputs(cfg, 2)
    L = O.lib()
    v = inp["wu"].view(np.float16).astype(np.float32).reshape(-1)[:4096]
    enc = np.array([L.oracle_e4m3(float(t)) for t in v], np.uint8)
    assert np.array_equal(enc, inp["wu_q"].reshape(-1)[:4096])


@pytest.mark.parametrize("bf16", [False, True])
def test_rmsnorm_oracle_matches_numpy_restatement(bf16):
    """Pre-MoE RMSNorm order: lane-strided 8-element chunks with fmaf, xor
    butterfly, r = sqrt(ss / d + eps), xn = round16((x * g) / r)."""
    rng = np.random.default_rng(5)
    d, T = 512, 3
    v = rng.standard_normal((T, d)).astype(np.float32)
    gv = (1 + 0.1 * rng.standard_normal(d)).astype(np.float32)
    to16 = (lambda a: (a.view(np.uint32) >> 16).astype(np.uint16)) if bf16 else \
        (lambda a: a.astype(np.float16).view(np.uint16))
    x, g = to16(v), to16(gv)
    out = O.rmsnorm(x, g, 1e-5, bf16)
    f = (lambda u: (u.astype(np.uint32) << 16).view(np.float32)) if bf16 else \
        (lambda u: u.view(np.float16).astype(np.float32))
    xf, gf = f(x), f(g)
    for t in range(T):
        p = []
        for lane in range(32):
            acc = np.float32(0)
            for c in range(lane, d // 8, 32):
                for j in range(8 * c, 8 * c + 8):
                    acc = np.float32(np.float64(acc) + np.float64(xf[t, j]) * np.float64(xf[t, j]))
            p.append(acc)
        for off in (16, 8, 4, 2, 1):
            p = [np.float32(p[i] + p[i ^ off]) for i in range(32)]
        r = np.float32(np.sqrt(np.float32(np.float32(p[0] / np.float32(d)) + np.float32(1e-5))))
        q = ((xf[t] * gf) / r).astype(np.float32)
        if bf16:   # round to nearest even
            u = q.view(np.uint32).astype(np.uint64)
            ref = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
        else:
            ref = q.astype(np.float16).view(np.uint16)
        assert np.array_equal(out[t], ref)


def test_residual_starts_the_combine():
    """With a residual the combine is ((r + w0*y0) + w1*y1) ...; a zero
    residual leaves the output unchanged and a residual without kept routes
    is copied through."""
    cfg = sm.LayerConfig(1, 16, 256, 256, 8, 2, 0.5)
    inp = sm.make_inputs(cfg, 2)
    base = O.forward(inp, cfg, nthreads=2)["out"]
    zero = O.forward({**inp, "residual": np.zeros_like(inp["x"])}, cfg, nthreads=2)["out"]
    assert np.array_equal(base, zero)
    with_r = O.forward({**inp, "residual": inp["x"]}, cfg, nthreads=2)
    xr = inp["x"].view(np.float16).astype(np.float32)
    dropped = [t for t in range(cfg.T) if (with_r["route_slot"][t * 2:(t + 1) * 2] < 0).all()]
    for t in dropped:
        assert np.array_equal(with_r["out"][t], xr[t])
    np.testing.assert_allclose(with_r["out"], base + xr, rtol=1e-6, atol=1e-6)
