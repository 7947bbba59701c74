"""Camera-sharded DFA on 2 GPUs (NCCL): each rank samples 3 of the 6 cameras with the softmax
taken over all 6, the partial sums are all-reduced, and the result equals the single-GPU
layer.  Skipped unless 2 GPUs are visible."""
import os
import socket
import tempfile

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out_dir):
    import datetime
    import sys

    repo = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, repo)
    import torch.distributed as dist

    from sparse4d_tt_b200 import DeformableFeatureAggregation, ops
    from sparse4d_tt_b200 import synthetic as syn

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dev = torch.device(f"cuda:{rank}")
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        cfg = syn.DFAConfig(bs=2, num_anchor=900)
        ins = syn.make_inputs(cfg, 41)
        params = syn.make_params(cfg, torch.Generator().manual_seed(42))
        packed = ops.pack_feature_maps([m.to(dev) for m in ins.feature_maps], dtype=torch.float32)
        args = (ins.instance_feature.to(dev), ins.anchor.to(dev), ins.anchor_embed.to(dev), packed,
                ins.projection_mat.to(dev), ins.image_wh.to(dev), cfg.spatial_shapes, 2, 900)
        sharded = DeformableFeatureAggregation(dev, params, {"FEATURE_DTYPE": torch.float32},
                                               mesh_device=dist.group.WORLD).run(*args)
        single = DeformableFeatureAggregation(dev, params, {"FEATURE_DTYPE": torch.float32}).run(*args)
        torch.cuda.synchronize()
        np.save(os.path.join(out_dir, f"err{rank}.npy"), np.array((sharded - single).abs().max().item()))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_camera_sharded_layer_matches_single_gpu():
    out_dir = tempfile.mkdtemp()
    mp.start_processes(_worker, args=(2, _free_port(), out_dir), nprocs=2, start_method="spawn")
    for r in range(2):
        assert float(np.load(os.path.join(out_dir, f"err{r}.npy"))) <= 1e-5
