"""Camera-sharded DFA host logic on 2 CPU ranks (gloo).  The per-rank partial sums come from
the numpy oracle (test infrastructure standing in for the CUDA gather, which needs a GPU); the
product code under test is ``camera_shard``: the camera split, the combining collectives and
the frame x camera process grid."""
import os
import socket
import tempfile

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _case(seed=0, bs=2, A=24, nc=6, P=13, G=8):
    rng = np.random.default_rng(seed)
    shapes = [(8, 20), (4, 10), (2, 5), (1, 3)]
    maps = [rng.standard_normal((bs, nc, 256, h, w)).astype(np.float32) for h, w in shapes]
    uv = (rng.random((bs, A, nc, P, 2)) * 1.4 - 0.2).astype(np.float32)
    logits = (rng.standard_normal((bs, A, nc, len(shapes), P, G)) * 2).astype(np.float32)
    return maps, uv, logits


def _worker(rank, world, port, out_dir):
    import sys

    repo = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, repo)
    import torch.distributed as dist

    from oracle import dfa_numpy as onp
    from sparse4d_tt_b200 import camera_shard as cs

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        maps, uv, logits = _case()
        feat, shape, start = onp.pack_feature_maps(maps)
        full = onp.deformable_aggregation(feat, shape, start, uv, logits)
        cb, ce = cs.rank_camera_range(6)
        part = torch.from_numpy(onp.deformable_aggregation(feat, shape, start, uv, logits, cam_range=(cb, ce)))
        summed = cs.reduce_partial_sums(part.clone())
        scattered = cs.reduce_partial_sums(part.clone(), scatter=True)
        rows = cs.reduce_partial_sums(part.reshape(-1, 256).clone(), scatter=True)
        rb, re_ = cs.shard_rows(part.shape[0] * part.shape[1])
        grid = cs.make_groups(world, world)
        res = {
            "range": np.array([cb, ce]),
            "allreduce_err": np.array((summed.numpy() - full).__abs__().max()),
            "scatter_err": np.array((scattered.numpy() - full[:, rank * 12:(rank + 1) * 12]).__abs__().max()),
            "rows": np.array([rb, re_]),
            "rows_err": np.array((rows.numpy() - full.reshape(-1, 256)[rb:re_]).__abs__().max()),
            "grid": np.array([grid[0], dist.get_world_size(grid[1])]),
        }
        np.savez(os.path.join(out_dir, f"rank{rank}.npz"), **res)
    finally:
        dist.destroy_process_group()


def test_camera_sharded_partial_sums_two_ranks():
    out_dir = tempfile.mkdtemp()
    mp.start_processes(_worker, args=(2, _free_port(), out_dir), nprocs=2, start_method="spawn")
    r0 = np.load(os.path.join(out_dir, "rank0.npz"))
    r1 = np.load(os.path.join(out_dir, "rank1.npz"))
    assert r0["range"].tolist() == [0, 3] and r1["range"].tolist() == [3, 6]
    for r in (r0, r1):
        assert float(r["allreduce_err"]) <= 1e-5  # global softmax over all 6 cameras
        assert float(r["scatter_err"]) <= 1e-5
        assert float(r["rows_err"]) <= 1e-5
        assert r["grid"].tolist() == [0, 2]
    assert r0["rows"].tolist() == [0, 24] and r1["rows"].tolist() == [24, 48]  # whole frames (bs 2)


def _grid_worker(rank, world, port, out_dir):
    """4 ranks as 2 frame groups x 2 camera halves: each rank takes its frame group's frames
    and its camera half, the partial sums meet by a row reduce-scatter inside the camera group."""
    import datetime
    import sys

    repo = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, repo)
    import torch.distributed as dist

    from oracle import dfa_numpy as onp
    from sparse4d_tt_b200 import camera_shard as cs

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        maps, uv, logits = _case(seed=5, bs=4, A=10)
        feat, shape, start = onp.pack_feature_maps(maps)
        full = onp.deformable_aggregation(feat, shape, start, uv, logits).reshape(4, 10, 256)
        fgroup, cgroup = cs.make_groups(world, 2)
        frames = slice(2 * fgroup, 2 * fgroup + 2)
        cb, ce = cs.rank_camera_range(6, cgroup)
        part = onp.deformable_aggregation(feat[frames], shape, start, uv[frames], logits[frames], cam_range=(cb, ce))
        rows = cs.reduce_partial_sums(torch.from_numpy(part).reshape(-1, 256).contiguous(), cgroup, scatter=True)
        rb, re_ = cs.shard_rows(20, cgroup)
        want = full[frames].reshape(-1, 256)[rb:re_]
        np.savez(os.path.join(out_dir, f"grid{rank}.npz"), fgroup=np.array(fgroup), cams=np.array([cb, ce]),
                 rows=np.array([rb, re_]), err=np.array(np.abs(rows.numpy() - want).max()))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_frame_by_camera_grid_four_ranks():
    out_dir = tempfile.mkdtemp()
    mp.start_processes(_grid_worker, args=(4, _free_port(), out_dir), nprocs=4, start_method="spawn")
    got = [np.load(os.path.join(out_dir, f"grid{r}.npz")) for r in range(4)]
    assert [int(g["fgroup"]) for g in got] == [0, 0, 1, 1]
    assert [g["cams"].tolist() for g in got] == [[0, 3], [3, 6], [0, 3], [3, 6]]
    assert [g["rows"].tolist() for g in got] == [[0, 10], [10, 20], [0, 10], [10, 20]]
    for g in got:
        assert float(g["err"]) <= 1e-5


def test_camera_split_shapes():
    from sparse4d_tt_b200.camera_shard import camera_split

    assert camera_split(6, 2) == [(0, 3), (3, 6)]
    assert camera_split(6, 4) == [(0, 2), (2, 4), (4, 5), (5, 6)]
    assert camera_split(6, 8)[6:] == [(6, 6), (6, 6)]
    with pytest.raises(ValueError):
        camera_split(6, 0)


def test_local_softmax_differs_from_global():
    """The reference's mesh mode normalises over each device's own cameras
    (model/sparse4d_head.py:93), which is not the single-device result; the global softmax
    used here is."""
    from oracle import dfa_numpy as onp

    maps, uv, logits = _case(3)
    feat, shape, start = onp.pack_feature_maps(maps)
    full = onp.deformable_aggregation(feat, shape, start, uv, logits)
    local = sum(onp.deformable_aggregation(feat[:, :], shape[c0:c1], start[c0:c1], uv[:, :, c0:c1],
                                           logits[:, :, c0:c1]) for c0, c1 in ((0, 3), (3, 6)))
    assert np.abs(local - full).max() > 1e-3
