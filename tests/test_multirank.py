"""Row sharding across ranks, on CPU with world-size-2 gloo process groups.

Each rank cuts its rows out of a tensor (hxq_b200.shard.slice_rows, the
same rows hxq_b200.sharded.ShardedDecompress gives a rank), decompresses
them with the oracle, and the ranks gather weights and sums of squared
sidecar deltas.  Rank 0 checks the reassembled matrix is bit-identical to
the whole-tensor result and that the combined confidence
(sharded.combine_sumsq) equals the exact one.  The column-split matmul's
output assembly (sharded.assemble_gathered) is checked the same way, and
the driver's launch grouping and offsets on their own.
"""
import os
import socket

import numpy as np
import pytest

WORLD = 2


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, kind: str, q):
    import sys
    repo = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, repo)
    sys.path.insert(0, os.path.join(repo, "hxq-native_b200"))
    import torch.distributed as dist
    from datetime import timedelta

    from hxq_b200 import synth
    from hxq_b200.shard import shard_rows, slice_rows
    from hxq_b200.sharded import combine_sumsq
    from oracle.oracle import Oracle

    dist.init_process_group("gloo", rank=rank, world_size=world, init_method=f"tcp://127.0.0.1:{port}",
                            timeout=timedelta(seconds=60))
    try:
        d = synth.vq12(1376 * 2 + 5, 256, 77, frac=0.02) if kind == "vq12" else \
            synth.scalar(301, 96, 78, frac=0.05)
        # a few entries the reference skips, to check the cut drops them too
        d["rows"] = np.concatenate([d["rows"], np.array([d["out_f"], 3], np.uint32)])
        d["cols"] = np.concatenate([d["cols"], np.array([1, d["in_f"] + 2], np.uint32)])
        d["vals"] = np.concatenate([d["vals"], np.array([9.0, 9.0], np.float32)])
        orc = Oracle()
        r0, r1 = shard_rows(d["out_f"], rank, world)
        part = slice_rows(d, r0, r1)
        err, w, _ = orc.decompress(part)
        ss = orc.l2_exact(part) ** 2
        got_w = [None] * world
        got_ss = [None] * world
        dist.all_gather_object(got_w, (r0, r1, err, w))
        dist.all_gather_object(got_ss, ss)
        if rank == 0:
            e_full, w_full, _ = orc.decompress(d)
            pieces = sorted(got_w, key=lambda t: t[0])
            assert pieces[0][0] == 0 and pieces[-1][1] == d["out_f"]
            assert all(p[2] == 0 for p in pieces)
            whole = np.concatenate([p[3] for p in pieces])
            ok_w = np.array_equal(whole.view(np.uint32), w_full.view(np.uint32))
            exact = orc.l2_exact(d)
            conf = combine_sumsq(got_ss)
            ok_c = abs(conf - exact) <= 1e-6 * exact
            q.put((ok_w, ok_c, conf, exact))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("kind", ["vq12", "scalar"])
def test_row_shards_gloo_world2(kind):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, WORLD, port, kind, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    ok_w, ok_c, conf, exact = q.get(timeout=10)
    assert ok_w, "reassembled shards differ from the whole-tensor decompress"
    assert ok_c, (conf, exact)


def test_shard_rows_partition():
    from hxq_b200.shard import shard_rows
    for out_f in (1, 7, 4096, 11008):
        for world in (1, 2, 3, 4, 8):
            spans = [shard_rows(out_f, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == out_f
            assert all(spans[i][1] == spans[i + 1][0] for i in range(world - 1))


def _matmul_worker(rank: int, world: int, port: int, q):
    """Column-split fused matmul: each rank owns the output features of its
    row shard, computes them with the oracle (the reference decompress of its
    rows, then the ordered matmul) and the ranks all-gather [ranks, N, rows];
    rank 0 checks the permuted result is bit-identical to the whole-tensor
    product."""
    import sys
    repo = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, repo)
    sys.path.insert(0, os.path.join(repo, "hxq-native_b200"))
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    from hxq_b200 import synth
    from hxq_b200.shard import shard_rows, slice_rows
    from hxq_b200.sharded import assemble_gathered
    from oracle.oracle import Oracle

    dist.init_process_group("gloo", rank=rank, world_size=world, init_method=f"tcp://127.0.0.1:{port}",
                            timeout=timedelta(seconds=60))
    try:
        out_f, in_f, N = 1376 * 2, 256, 3        # an even split, as the 7B shapes are
        d = synth.vq12(out_f, in_f, 91, frac=0.02)
        _, x = synth.activations(N, in_f, 92)
        orc = Oracle()
        r0, r1 = shard_rows(out_f, rank, world)
        part = slice_rows(d, r0, r1)
        err, w, _ = orc.decompress(part)
        y = torch.from_numpy(orc.dense_matmul(x, w.reshape(r1 - r0, in_f)))
        g = torch.empty((world * N, r1 - r0), dtype=torch.float32)
        dist.all_gather_into_tensor(g, y)
        if rank == 0:
            whole = assemble_gathered(g, world, N, r1 - r0).numpy()
            e_full, w_full, _ = orc.decompress(d)
            ref = orc.dense_matmul(x, w_full.reshape(out_f, in_f))
            q.put((err == 0 and e_full == 0, bool(np.array_equal(whole.view(np.uint32), ref.view(np.uint32)))))
    finally:
        dist.destroy_process_group()


def test_column_split_matmul_gloo_world2():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_matmul_worker, args=(r, WORLD, port, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    ok_err, ok_y = q.get(timeout=10)
    assert ok_err
    assert ok_y, "gathered output shards differ from the whole-matrix product"


def test_launch_groups_and_offsets():
    from hxq_b200.sharded import MAX_LAYERS_PER_LAUNCH, launch_groups, packed_offsets
    for nl in (1, 5, 32):
        for world in (1, 2, 3, 8, 16):
            groups = launch_groups(nl, world)
            flat = [layer for g in groups for layer in g]
            assert flat == list(range(nl))
            per = min(MAX_LAYERS_PER_LAUNCH, world, nl)
            assert all(len(g) == per for g in groups[:-1]) and 1 <= len(groups[-1]) <= per
    offs, total = packed_offsets([5, 0, 7])
    assert offs == [0, 5, 5] and total == 12


def test_assemble_gathered_numpy_and_torch():
    import torch

    from hxq_b200.sharded import assemble_gathered
    world, N, rows = 3, 2, 4
    full = np.arange(N * world * rows, dtype=np.float32).reshape(N, world * rows)
    shards = [full[:, r * rows:(r + 1) * rows] for r in range(world)]
    g = np.concatenate(shards, axis=0)                      # [world * N, rows]
    assert np.array_equal(assemble_gathered(g, world, N, rows), full)
    assert torch.equal(assemble_gathered(torch.from_numpy(g), world, N, rows), torch.from_numpy(full))
