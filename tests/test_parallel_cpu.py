"""CPU checks of the tensor-parallel plan (kotensor_b200/parallel.py): shard
bounds, host shards against quantizing the sliced fp32 weight, and the
row-/column-parallel products reassembled by gloo collectives over two CPU
processes, with the oracle computing each rank's part."""
import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")


def test_shard_bounds_cover_align_and_reject(kt):
    from kotensor_b200 import parallel as P
    for extent, g in [(4096, 64), (960, 96), (130, 64), (14336, 64), (7, 1)]:
        groups = (extent + g - 1) // g
        for parts in (1, 2, 3, 8):
            if parts > groups:
                with pytest.raises(ValueError):
                    [P.shard_bounds(P.ROWS, extent, g, parts, i) for i in range(parts)]
                continue
            b = [P.shard_bounds(P.ROWS, extent, g, parts, i) for i in range(parts)]
            assert b[0][0] == 0 and b[-1][1] == extent
            assert all(b[i][1] == b[i + 1][0] for i in range(parts - 1))
            assert all(x % g == 0 for x, _ in b)
    for extent in (14336, 1537, 9):
        for parts in (1, 2, 3, 8):
            b = [P.shard_bounds(P.COLUMNS, extent, 64, parts, i) for i in range(parts)]
            assert b[0][0] == 0 and b[-1][1] == extent and all(b[i][1] == b[i + 1][0] for i in range(parts - 1))
    for bad in [(P.ROWS, 64, 64, 0, 0), (P.ROWS, 64, 64, 2, 2), (2, 64, 64, 1, 0), (P.COLUMNS, 0, 64, 1, 0)]:
        with pytest.raises(ValueError):
            P.shard_bounds(*bad)


@pytest.mark.parametrize("bits,g", [(4, 64), (4, 32), (8, 64)])
@pytest.mark.parametrize("shape", [(256, 1537), (640, 96), (130, 33)])
@pytest.mark.parametrize("parts", [2, 3])
def test_host_shards_are_the_quantized_slices(kt, oracle, bits, g, shape, parts):
    from kotensor_b200 import parallel as P
    rng = np.random.default_rng(sum(shape) + bits + g + parts)
    w = (rng.standard_normal(shape, dtype=np.float32) * 0.05).astype(np.float32)
    full = oracle.quantize(w, bits, g)
    for axis in (P.ROWS, P.COLUMNS):
        extent = shape[axis]
        if axis == P.ROWS and parts > (extent + g - 1) // g:
            continue
        for i in range(parts):
            b, e = P.shard_bounds(axis, extent, g, parts, i)
            q, s, z, sh = P.shard_host(full.qdata, full.scales, full.zeros, shape, bits, g, axis, parts, i)
            ref = oracle.quantize(w[b:e] if axis == P.ROWS else np.ascontiguousarray(w[:, b:e]), bits, g)
            assert sh == ((e - b, shape[1]) if axis == P.ROWS else (shape[0], e - b))
            assert np.array_equal(q.reshape(-1), ref.qdata.reshape(-1))
            assert np.array_equal(s.reshape(-1).view(np.uint32), ref.scales.reshape(-1).view(np.uint32))
            if bits == 4:
                assert np.array_equal(z.reshape(-1), ref.zeros.reshape(-1))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _tp_rank(rank, world, port, out_dir):
    import torch.distributed as dist
    from kotensor_b200 import parallel as P
    from oracle import oracle as O
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        rng = np.random.default_rng(7)
        k, n, g, m = 512, 300, 64, 3
        w = (rng.standard_normal((k, n), dtype=np.float32) * 0.02).astype(np.float32)
        x = rng.standard_normal((m, k), dtype=np.float32)
        bias = rng.standard_normal(n, dtype=np.float32)
        full = O.quantize(w, 4, g)
        # row-parallel: partial products of this rank's K-slice, summed across ranks, bias once
        b, e = P.shard_bounds(P.ROWS, k, g, world, rank)
        q, s, z, sh = P.shard_host(full.qdata, full.scales, full.zeros, (k, n), 4, g, P.ROWS, world, rank)
        part = O.multiply_quantized(np.ascontiguousarray(x[:, b:e]), O.OracleQTensor(q.reshape(-1), s.reshape(-1), z.reshape(-1), sh[0], sh[1], 4, g), threads=2)
        t = torch.from_numpy(part.astype(np.float32))
        dist.all_reduce(t)
        y_row = t.numpy() + bias[None, :]
        # column-parallel: this rank's columns, gathered in rank order
        b, e = P.shard_bounds(P.COLUMNS, n, g, world, rank)
        q, s, z, sh = P.shard_host(full.qdata, full.scales, full.zeros, (k, n), 4, g, P.COLUMNS, world, rank)
        ycol = O.multiply_quantized(x, O.OracleQTensor(q.reshape(-1), s.reshape(-1), z.reshape(-1), sh[0], sh[1], 4, g), threads=2)
        parts = [None] * world
        dist.all_gather_object(parts, ycol)
        y_col = np.concatenate(parts, axis=1)
        # column-parallel greedy argmax: each rank's best (value, global column) pair,
        # gathered, merged in rank order (larger value, then lower column)
        lg = rng.standard_normal((4, 90), dtype=np.float32)
        lg[0, 5] = lg[0, 80] = 9.0   # a tie across the shard boundary
        lg[1] = -3e9                 # nothing above -1e9: column 0
        lg[2, 89] = 9.0              # the last column
        b, e = P.shard_bounds(P.COLUMNS, 90, 1, world, rank)
        pairs = []
        for row in lg[:, b:e]:
            best, idx = np.float32(-1e9), None
            for j, v in enumerate(row):
                if v > best:
                    best, idx = v, b + j
            pairs.append((best, idx))
        every = [None] * world
        dist.all_gather_object(every, pairs)
        tokens = []
        for r in range(lg.shape[0]):
            best, idx = np.float32(-1e9), None
            for p in range(world):
                v, i = every[p][r]
                if i is not None and (v > best or (v == best and i < idx)):
                    best, idx = v, i
            tokens.append(0 if idx is None else idx)
        if rank == 0:
            masked = np.where(lg > np.float32(-1e9), lg, -np.inf)
            want = [int(np.argmax(m)) if np.isfinite(m).any() else 0 for m in masked]
            np.save(os.path.join(out_dir, "argmax.npy"), np.array([tokens, want]))
            ref = O.multiply_quantized(x, full, threads=2)
            np.save(os.path.join(out_dir, "ref.npy"), ref)
            np.save(os.path.join(out_dir, "row.npy"), y_row - bias[None, :])
            np.save(os.path.join(out_dir, "col.npy"), y_col)
    finally:
        dist.destroy_process_group()


def test_tensor_parallel_plan_with_gloo(kt, oracle, tmp_path):
    import torch.multiprocessing as mp
    mp.spawn(_tp_rank, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True)
    ref = np.load(tmp_path / "ref.npy")
    scale = np.abs(ref).max()
    assert np.abs(np.load(tmp_path / "row.npy") - ref).max() <= 1e-5 * scale
    assert np.abs(np.load(tmp_path / "col.npy") - ref).max() <= 1e-5 * scale
    tokens, want = np.load(tmp_path / "argmax.npy")
    assert np.array_equal(tokens, want) and want[0] == 5 and want[1] == 0 and want[2] == 89


TP_DECODER = dict(vocab=384, dim=256, layers=2, heads=8, kv_heads=4, hidden=512, rope_theta=500000.0,
                  rope_scaling=(8.0, 1.0, 4.0, 8192), bits=4, group_size=64, tied=False, qkv_bias=True)


def _tp_decoder_rank(rank, world, port, out_dir):
    """One rank of the tensor-parallel decode step of kotensor_b200/decoder.py
    restated with the oracle: this rank's heads, hidden block and vocabulary
    columns (tensor_parallel_plan), each shard quantized from its slice of the
    fp32 weight, the two row-parallel partial sums per layer all-reduced over
    gloo, and the greedy token merged across ranks by (value, lowest column)."""
    import math
    import torch.distributed as dist
    from kotensor_b200 import decoder as D
    from oracle import decoder_oracle as DO
    from oracle import oracle as O
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        cfg = DO.DecoderConfig(**TP_DECODER)
        plan = D.tensor_parallel_plan(D.DecoderConfig(**TP_DECODER), world, rank)
        q0, q1 = plan["q"]
        k0, k1 = plan["kv"]
        h0, h1 = plan["hidden"]
        v0, v1 = plan["vocab"]
        rng = np.random.default_rng(31)
        hd, kv = cfg.head_dim, cfg.kv_heads * cfg.head_dim

        def fp(k, n):
            return (rng.standard_normal((k, n), dtype=np.float32) * np.float32(0.02)).astype(np.float32)

        def q(w):
            return O.quantize(np.ascontiguousarray(w), cfg.bits, cfg.group_size)

        full, mine = [], []
        for _ in range(cfg.layers):
            w = {"wq": fp(cfg.dim, cfg.dim), "wk": fp(cfg.dim, kv), "wv": fp(cfg.dim, kv), "wo": fp(cfg.dim, cfg.dim),
                 "wg": fp(cfg.dim, cfg.hidden), "wu": fp(cfg.dim, cfg.hidden), "wd": fp(cfg.hidden, cfg.dim)}
            b = {"bq": fp(1, cfg.dim)[0], "bk": fp(1, kv)[0], "bv": fp(1, kv)[0], "bo": fp(1, cfg.dim)[0],
                 "bg": np.zeros(cfg.hidden, np.float32), "bu": np.zeros(cfg.hidden, np.float32),
                 "bd": fp(1, cfg.dim)[0]}
            n = {"norm1": (1 + fp(1, cfg.dim)[0] * 5).astype(np.float32),
                 "norm2": (1 + fp(1, cfg.dim)[0] * 5).astype(np.float32)}
            full.append({**{k: q(v) for k, v in w.items()}, **b, **n})
            mine.append({"wq": q(w["wq"][:, q0:q1]), "wk": q(w["wk"][:, k0:k1]), "wv": q(w["wv"][:, k0:k1]),
                         "wo": q(w["wo"][q0:q1]), "wg": q(w["wg"][:, h0:h1]), "wu": q(w["wu"][:, h0:h1]),
                         "wd": q(w["wd"][h0:h1]), "bq": b["bq"][q0:q1], "bk": b["bk"][k0:k1],
                         "bv": b["bv"][k0:k1], "bo": b["bo"], "bd": b["bd"], **n})
        emb_f = (rng.standard_normal((cfg.vocab, cfg.dim), dtype=np.float32) * np.float32(0.5)).astype(np.float32)
        head_f = fp(cfg.dim, cfg.vocab)
        final = (1 + fp(1, cfg.dim)[0] * 5).astype(np.float32)
        emb, head = q(emb_f), q(head_f)
        head_mine = q(head_f[:, v0:v1])
        ref = DO.OracleDecoder(DO.DecoderWeights(cfg, emb, full, final, head, np.zeros(cfg.vocab, np.float32)), 16)
        heads_l, kv_l = plan["heads"], plan["kv_heads"]
        group = cfg.heads // cfg.kv_heads
        keys = np.zeros((cfg.layers, kv_l, 16, hd), np.float32)
        values = np.zeros_like(keys)
        freqs = DO.inv_freq(hd, cfg.rope_theta, cfg.rope_scaling)
        scale = np.float32(1.0) / np.float32(math.sqrt(float(hd)))

        def all_reduce(a):
            t = torch.from_numpy(np.ascontiguousarray(a, np.float32))
            dist.all_reduce(t)
            return t.numpy()

        out, token = [], 3
        for pos in range(6):
            x = emb.dequantize_row(token).astype(np.float32)
            for l, L in enumerate(mine):
                n1 = DO._rmsnorm(x, L["norm1"], cfg.eps)
                qv = DO._rope(DO._linear(n1, L["wq"], L["bq"]), hd, freqs, pos)
                kk = DO._rope(DO._linear(n1, L["wk"], L["bk"]), hd, freqs, pos)
                vv = DO._linear(n1, L["wv"], L["bv"])
                keys[l, :, pos] = kk.reshape(kv_l, hd)
                values[l, :, pos] = vv.reshape(kv_l, hd)
                ctx = np.empty(heads_l * hd, np.float32)
                for h in range(heads_l):  # local head h uses local kv head h // group
                    sc = (keys[l, h // group, :pos + 1] @ qv[h * hd:(h + 1) * hd]).astype(np.float32) * scale
                    e = np.exp((sc - max(np.float32(-1e9), sc.max())).astype(np.float64)).astype(np.float32)
                    wts = e * (np.float32(1.0) / np.sum(e, dtype=np.float32))
                    ctx[h * hd:(h + 1) * hd] = wts @ values[l, h // group, :pos + 1]
                part = O.multiply_quantized(ctx.reshape(1, -1), L["wo"]).reshape(-1)
                x = (x + all_reduce(part) + L["bo"]).astype(np.float32)
                n2 = DO._rmsnorm(x, L["norm2"], cfg.eps)
                gate = DO._linear(n2, L["wg"], np.zeros(h1 - h0, np.float32))
                up = DO._linear(n2, L["wu"], np.zeros(h1 - h0, np.float32))
                act = (gate / (np.float32(1.0) + np.exp(-gate.astype(np.float64)).astype(np.float32)) * up)
                part = O.multiply_quantized(act.astype(np.float32).reshape(1, -1), L["wd"]).reshape(-1)
                x = (x + all_reduce(part) + L["bd"]).astype(np.float32)
            logits = DO._linear(DO._rmsnorm(x, final, cfg.eps), head_mine, np.zeros(v1 - v0, np.float32))
            best = max(range(v1 - v0), key=lambda j: (logits[j], -j))
            pairs = [None] * world
            dist.all_gather_object(pairs, (float(logits[best]), v0 + best, logits))
            token = min(((-v, c) for v, c, _ in pairs))[1]
            out.append((np.concatenate([p[2] for p in pairs]), token))
        if rank == 0:
            ref_out, tok = [], 3
            for pos in range(6):
                lg = ref.step(tok)
                ref_out.append(lg)
                tok = out[pos][1]
            np.save(os.path.join(out_dir, "tp_dec.npy"),
                    np.array([(o[0], r, o[1], DO.argmax(r)) for o, r in zip(out, ref_out)], dtype=object),
                    allow_pickle=True)
    finally:
        dist.destroy_process_group()


def test_tensor_parallel_decoder_plan_with_gloo(kt, oracle, tmp_path):
    """The tensor-parallel decode step over two CPU ranks equals the unsharded
    oracle step within float32 rounding, and its greedy token is the oracle's."""
    import torch.multiprocessing as mp
    mp.spawn(_tp_decoder_rank, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True)
    for whole, ref, token, best in np.load(tmp_path / "tp_dec.npy", allow_pickle=True):
        assert np.abs(whole - ref).max() <= 1e-4 * np.abs(ref).max()
        assert token == best


def test_tensor_parallel_plan_rejects_bad_splits(kt):
    from kotensor_b200 import decoder as D
    cfg = D.DecoderConfig(**TP_DECODER)
    plans = [D.tensor_parallel_plan(cfg, 4, r) for r in range(4)]
    assert [p["q"] for p in plans] == [(0, 64), (64, 128), (128, 192), (192, 256)]
    assert [p["kv"] for p in plans] == [(0, 32), (32, 64), (64, 96), (96, 128)]
    assert plans[-1]["hidden"][1] == cfg.hidden and plans[0]["vocab"][0] == 0
    with pytest.raises(ValueError):
        D.tensor_parallel_plan(cfg, 3, 0)  # 8 heads over 3 ranks
    with pytest.raises(ValueError):
        D.tensor_parallel_plan(cfg, 8, 0)  # 32 output-projection rows per rank, groups of 64
