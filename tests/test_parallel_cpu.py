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
