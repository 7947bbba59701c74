"""CPU restatement of the reference's InstanceBank (inference): temporal projection of the cached
anchors (``get``), the top-300 merge of new instances with the 600 cached ones (``update``) and
the confidence-decayed top-600 cache (``cache``) -- ``model/instance_bank.py:95-306`` with the
projection of ``InstanceBank._anchor_projection`` (``model/instance_bank.py:322-369``).

TEST INFRASTRUCTURE ONLY: the tests, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU
baseline use it as the checker; the product path (``sparse4d_tt_b200.instance_bank``) runs the
CUDA kernels and never calls this module.

Top-k order: scores descending, equal scores by ascending anchor index (a stable sort).  The
reference's ``ttnn.topk`` (un-vendored tt-metal) leaves the order of equal scores unspecified;
with real-valued confidences ties have measure zero, and the tests compare tie-free inputs
against ``torch.topk`` as well.
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch

X, Y, Z = 0, 1, 2
W, L, H = 3, 4, 5
SIN_YAW, COS_YAW = 6, 7
VX, VY, VZ = 8, 9, 10


def anchor_projection(anchor: torch.Tensor, T_src2dst: torch.Tensor, time_interval: Optional[torch.Tensor]):
    """``[bs, N, 11]`` anchors moved by ``-velocity * time_interval`` and transformed by
    ``T_src2dst [bs, 4, 4]`` (``model/instance_bank.py:322-369``).  The output keeps the
    reference's yaw order: the rotated ``[cos, sin]`` pair lands in the (sin, cos) slots."""
    vel = anchor[..., VX:]
    T = T_src2dst.unsqueeze(1).to(anchor.dtype)
    center = anchor[..., [X, Y, Z]]
    if time_interval is not None:
        center = center - vel * time_interval.to(vel.dtype)[:, None, None]
    center = torch.matmul(T[..., :3, :3], center[..., None]).squeeze(-1) + T[..., :3, 3]
    size = anchor[..., [W, L, H]]
    yaw = torch.matmul(T[..., :2, :2], anchor[..., [COS_YAW, SIN_YAW], None]).squeeze(-1)
    vel = torch.matmul(T[..., :3, :3], vel[..., None]).squeeze(-1)
    return torch.cat([center, size, yaw, vel], dim=-1)


def topk_stable(scores: torch.Tensor, k: int) -> Tuple[torch.Tensor, torch.Tensor]:
    """Top-k along the last dim: values descending, ties by ascending index."""
    order = torch.sort(scores, dim=-1, descending=True, stable=True).indices[..., :k]
    return torch.gather(scores, -1, order), order


def gather_rows(x: torch.Tensor, idx: torch.Tensor) -> torch.Tensor:
    return torch.gather(x, 1, idx[..., None].expand(-1, -1, x.shape[-1]))


class InstanceBankOracle:
    """Same flow as the reference class, on CPU tensors in fp32."""

    def __init__(self, anchor_data, instance_feature_data, num_anchor=900, embed_dims=256, num_temp_instances=600,
                 default_time_interval=0.5, confidence_decay=0.6, max_time_interval=2.0):
        self.anchor_data = anchor_data.float()
        self.instance_feature_data = instance_feature_data.float()
        self.num_anchor, self.embed_dims = num_anchor, embed_dims
        self.num_temp_instances = num_temp_instances
        self.default_time_interval = default_time_interval
        self.confidence_decay = confidence_decay
        self.max_time_interval = max_time_interval
        self.reset()

    def reset(self):
        self.cached_feature = self.cached_anchor = self.metas = self.mask = self.confidence = None

    def get(self, bs, metas):
        """``model/instance_bank.py:95-184``."""
        cached_feature = cached_anchor = None
        if self.cached_anchor is not None:
            ti = metas["timestamp"] - self.metas["timestamp"]
            self.mask = ti.abs() <= self.max_time_interval
            T = torch.stack([torch.as_tensor(x["T_global_inv"] @ self.metas["img_metas"][i]["T_global"],
                                             dtype=torch.float32) for i, x in enumerate(metas["img_metas"])])
            self.cached_anchor = anchor_projection(self.cached_anchor, T, -ti)
            cached_anchor = self.cached_anchor
            cached_feature = self.cached_feature
            ti = torch.where((ti != 0) & self.mask, ti, torch.tensor(self.default_time_interval, dtype=ti.dtype))
        else:
            self.reset()
            ti = torch.full((bs,), self.default_time_interval)
        inst = self.instance_feature_data[None].expand(bs, -1, -1)
        anchor = self.anchor_data[None].expand(bs, -1, -1)
        return inst, anchor, cached_feature, cached_anchor, ti

    def update(self, instance_feature, anchor, confidence):
        """``model/instance_bank.py:188-246``: the 300 most confident new instances after the
        600 cached ones, for the frames whose time gap is within ``max_time_interval``."""
        if self.cached_feature is None:
            return instance_feature, anchor
        n = self.num_anchor - self.num_temp_instances
        _, idx = topk_stable(confidence.max(dim=-1).values, n)
        feat = torch.cat([self.cached_feature, gather_rows(instance_feature, idx)], dim=1)
        anc = torch.cat([self.cached_anchor, gather_rows(anchor, idx)], dim=1)
        m = self.mask[:, None, None]
        return torch.where(m, feat, instance_feature), torch.where(m, anc, anchor)

    def cache(self, instance_feature, anchor, confidence, metas):
        """``model/instance_bank.py:248-306``."""
        if self.num_temp_instances <= 0:
            return
        self.metas = metas
        conf = confidence.max(dim=-1).values.double().sigmoid().float()  # sigmoid in double, rounded once
        if self.confidence is not None:
            k0 = self.num_temp_instances
            conf = torch.cat([torch.maximum(self.confidence * self.confidence_decay, conf[:, :k0]), conf[:, k0:]], -1)
        top, idx = topk_stable(conf, self.num_temp_instances)
        self.cached_feature = gather_rows(instance_feature, idx)
        self.cached_anchor = gather_rows(anchor, idx)
        self.confidence = top
