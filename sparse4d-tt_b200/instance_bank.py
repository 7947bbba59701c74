"""B200 InstanceBank (inference): the temporal instance cache that feeds the decoder 600 cached +
300 new anchors per frame, with the reference's interface (``model/instance_bank.py:34-306``:
``get`` / ``update`` / ``cache`` / ``reset``) and its per-frame flow:

* ``get(bs, metas)``: the cached anchors are moved to the current frame on the GPU
  (``s4d_instance_bank_project``); the transform ``T_global_inv @ T_global_prev`` and the time
  gap are formed on the host from ``metas``, as the reference does (``:116-128``);
* ``update(...)``: the 300 most confident new instances follow the 600 cached ones
  (``s4d_instance_bank_update``, one CTA per frame: score, sort, gather, merge);
* ``cache(...)``: the 600 most confident instances (sigmoid, decayed previous confidence) are
  kept for the next frame (``s4d_instance_bank_cache``).

All tensors live on the CUDA device; the kernels are in ``csrc/instance_bank.cu``.
"""
from __future__ import annotations

from typing import Dict, Optional

import numpy as np
import torch

from . import _lib as L
from . import ops

Tensor = torch.Tensor


def preprocess_instance_bank_parameters(pt_bank) -> Dict[str, Tensor]:
    """``model/instance_bank.py:372-387``: the learnable anchors and instance features."""
    return {"anchor_data": pt_bank.anchor.data.clone(),
            "instance_feature_data": pt_bank.instance_feature.data.clone()}


def project_anchors(anchor: Tensor, T_temp2cur: Tensor, time_interval: Optional[Tensor] = None,
                    out: Optional[Tensor] = None) -> Tensor:
    """``[bs, N, 11]`` anchors moved by ``-velocity * time_interval`` and transformed by
    ``T_temp2cur [bs, 4, 4]`` (``InstanceBank._anchor_projection``)."""
    name = "project_anchors"
    anchor = anchor.float().contiguous()
    T_temp2cur = T_temp2cur.float().contiguous()
    time_interval = None if time_interval is None else time_interval.float().contiguous()
    out = torch.empty_like(anchor) if out is None else out
    dev = ops._require_cuda(name, anchor, T_temp2cur, time_interval, out)
    bs, n, d = anchor.shape
    ops._require(d == 11 and tuple(T_temp2cur.shape) == (bs, 4, 4), f"{name}: anchor [bs, N, 11], T [bs, 4, 4]")
    ops._require(time_interval is None or tuple(time_interval.shape) == (bs,), f"{name}: time_interval [bs]")
    L.check(name, L.lib().s4d_instance_bank_project(anchor.data_ptr(), T_temp2cur.data_ptr(),
                                                    ops._ptr(time_interval), bs, n, out.data_ptr(),
                                                    ops._stream_ptr(dev)))
    return out


class InstanceBank:
    """Same constructor arguments, attributes and methods as the reference class; ``device`` is a
    CUDA device.  ``mesh_device`` is accepted for signature compatibility and ignored (every GPU
    keeps its own frames' bank)."""

    def __init__(self, device, anchor_data: Tensor, instance_feature_data: Tensor, num_anchor: int = 900,
                 embed_dims: int = 256, num_temp_instances: int = 600, default_time_interval: float = 0.5,
                 confidence_decay: float = 0.6, max_time_interval: float = 2.0, mesh_device=None) -> None:
        self.device = torch.device(device if not isinstance(device, int) else f"cuda:{device}")
        if self.device.type != "cuda":
            raise ValueError("InstanceBank runs on a CUDA device only")
        self.num_anchor, self.embed_dims = num_anchor, embed_dims
        self.num_temp_instances = num_temp_instances
        self.default_time_interval = default_time_interval
        self.confidence_decay = confidence_decay
        self.max_time_interval = max_time_interval
        self.anchor_data = anchor_data.float().to(self.device).contiguous()
        self.instance_feature_data = instance_feature_data.float().to(self.device).contiguous()
        self.reset()

    def reset(self) -> None:
        self.cached_feature = None
        self.cached_anchor = None
        self.metas = None
        self.mask = None  # [bs] bool (host), as the reference keeps it
        self.confidence = None
        self.instance_id = None
        self.prev_id = 0

    def get(self, bs: int, metas: dict):
        """Returns ``(instance_feature [bs, A, C], anchor [bs, A, 11], cached_feature,
        cached_anchor, time_interval [bs])`` (``model/instance_bank.py:95-184``)."""
        cached_feature = cached_anchor = None
        if self.cached_anchor is not None:
            ti = torch.as_tensor(metas["timestamp"], dtype=torch.float64) - torch.as_tensor(
                self.metas["timestamp"], dtype=torch.float64)
            ti = ti.float().reshape(bs)
            self.mask = ti.abs() <= self.max_time_interval
            T = torch.as_tensor(np.stack([x["T_global_inv"] @ self.metas["img_metas"][i]["T_global"]
                                          for i, x in enumerate(metas["img_metas"])]), dtype=torch.float32)
            self.cached_anchor = project_anchors(self.cached_anchor, T.to(self.device), (-ti).to(self.device))
            cached_anchor, cached_feature = self.cached_anchor, self.cached_feature
            ti = torch.where((ti != 0) & self.mask, ti, torch.tensor(self.default_time_interval))
        else:
            self.reset()
            ti = torch.full((bs,), self.default_time_interval)
        inst = self.instance_feature_data[None].expand(bs, -1, -1)
        anchor = self.anchor_data[None].expand(bs, -1, -1)
        return inst, anchor, cached_feature, cached_anchor, ti.to(self.device)

    def update(self, instance_feature: Tensor, anchor: Tensor, confidence: Tensor, bs: Optional[int] = None):
        """``[cached | top (A - num_temp) new]`` instances for the frames within the time limit
        (``model/instance_bank.py:188-246``)."""
        if self.cached_feature is None:
            return instance_feature, anchor
        name = "InstanceBank.update"
        feat, anc, conf = (t.float().contiguous() for t in (instance_feature, anchor, confidence))
        bs_, A, C = feat.shape
        out_f, out_a = torch.empty_like(feat), torch.empty_like(anc)
        mask = None if self.mask is None else self.mask.to(torch.uint8).to(self.device)
        ops._require(A == self.num_anchor, f"{name}: expected {self.num_anchor} anchors")
        L.check(name, L.lib().s4d_instance_bank_update(
            feat.data_ptr(), anc.data_ptr(), conf.data_ptr(), self.cached_feature.data_ptr(),
            self.cached_anchor.data_ptr(), ops._ptr(mask), bs_, A, conf.shape[-1], C, self.num_temp_instances,
            out_f.data_ptr(), out_a.data_ptr(), None, ops._stream_ptr(self.device)))
        return out_f, out_a

    def cache(self, instance_feature: Tensor, anchor: Tensor, confidence: Tensor, metas: dict,
              bs: Optional[int] = None) -> None:
        """Keeps the ``num_temp_instances`` most confident instances
        (``model/instance_bank.py:248-306``)."""
        if self.num_temp_instances <= 0:
            return
        name = "InstanceBank.cache"
        self.metas = metas
        feat, anc, conf = (t.float().contiguous() for t in (instance_feature, anchor, confidence))
        bs_, A, C = feat.shape
        K = self.num_temp_instances
        cf = torch.empty(bs_, K, C, device=self.device)
        ca = torch.empty(bs_, K, anc.shape[-1], device=self.device)
        cc = torch.empty(bs_, K, device=self.device)
        prev = None if self.confidence is None else self.confidence.contiguous()
        L.check(name, L.lib().s4d_instance_bank_cache(
            feat.data_ptr(), anc.data_ptr(), conf.data_ptr(), ops._ptr(prev), float(self.confidence_decay), bs_, A,
            conf.shape[-1], C, K, cf.data_ptr(), ca.data_ptr(), cc.data_ptr(), None, ops._stream_ptr(self.device)))
        self.cached_feature, self.cached_anchor, self.confidence = cf, ca, cc
