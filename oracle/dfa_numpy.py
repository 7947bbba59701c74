"""Numpy float32 restatement of the DFA path.  TEST INFRASTRUCTURE ONLY (see
``oracle/__init__.py``).

Independent of ``torch.nn.functional.grid_sample``: the bilinear taps are written out, on the
packed channels-last feature layout the CUDA operator reads (``[bs, Ncam * sum(HW), C]``
with per-(camera, level) ``spatial_shape`` and ``scale_start_index``).  It cross-checks the
torch oracle and states the operator's semantics at the operator boundary.

The keypoint projection evaluates every product and sum in one fixed order, without fused
multiply-add, so its depth mask, frustum mask and compacted indices are the integer
reference for the keypoint kernel (which uses the same order):

    size = exp(log_size); k = fix_scale * size  or  (sigmoid(logit) - 0.5) * size
    rx = cos*kx - sin*ky;  ry = sin*kx + cos*ky;  p = (rx + cx, ry + cy, kz + cz)
    X = ((P[r,0]*px + P[r,1]*py) + P[r,2]*pz) + P[r,3]      for r = 0, 1, 2
    mask = X2 > 1e-5;  z = X2 < 1e-5 ? 1e-5 : X2;  u = (X0 / z) / w;  v = (X1 / z) / h

which is the arithmetic of ``test/dfa_pcc.py:225-247`` (keypoints) and ``:322-333``
(projection), with the matrix products expanded term by term.
"""
from __future__ import annotations

import numpy as np

f32 = np.float32


def key_points(anchor: np.ndarray, logits: np.ndarray, fix_scale: np.ndarray) -> np.ndarray:
    """``[bs, A, P, 3]`` keypoints (``test/dfa_pcc.py:225-247``)."""
    anchor = anchor.astype(f32)
    bs, A = anchor.shape[:2]
    size = np.exp(anchor[..., 3:6])[:, :, None, :]  # [bs, A, 1, 3]
    fixed = fix_scale.astype(f32)[None, None] * size
    parts = [fixed]
    if logits is not None and logits.shape[-1] > 0:
        lg = logits.astype(f32).reshape(bs, A, -1, 3)
        sig = f32(1) / (f32(1) + np.exp(-lg))
        parts.append((sig - f32(0.5)) * size)
    k = np.concatenate(parts, axis=2)
    s = anchor[..., 6][:, :, None]
    c = anchor[..., 7][:, :, None]
    rx = c * k[..., 0] - s * k[..., 1]
    ry = s * k[..., 0] + c * k[..., 1]
    out = np.stack([rx + anchor[..., 0][:, :, None], ry + anchor[..., 1][:, :, None],
                    k[..., 2] + anchor[..., 2][:, :, None]], axis=-1)
    return out.astype(f32)


def project(kp: np.ndarray, proj: np.ndarray, image_wh: np.ndarray):
    """Project ``kp [bs, A, P, 3]`` with ``proj [bs, Ncam, 4, 4]``.

    Returns ``uv [bs, A, Ncam, P, 2]``, ``depth_mask [bs, A, Ncam, P]`` (bool) and
    ``visible [bs, A, Ncam, P]`` (bool)."""
    px = kp[:, :, None, :, 0]
    py = kp[:, :, None, :, 1]
    pz = kp[:, :, None, :, 2]
    P = proj.astype(f32)[:, None, :, None]  # [bs, 1, Ncam, 1, 4, 4]

    def row(r):
        return ((P[..., r, 0] * px + P[..., r, 1] * py) + P[..., r, 2] * pz) + P[..., r, 3]

    X0, X1, X2 = row(0), row(1), row(2)
    mask = X2 > f32(1e-5)
    z = np.where(X2 < f32(1e-5), f32(1e-5), X2).astype(f32)
    wh = image_wh.astype(f32)[:, None, :, None]  # [bs, 1, Ncam, 1, 2]
    u = (X0 / z) / wh[..., 0]
    v = (X1 / z) / wh[..., 1]
    vis = mask & (u >= 0) & (u <= 1) & (v >= 0) & (v <= 1)
    return np.stack([u, v], axis=-1).astype(f32), mask, vis


def pack_feature_maps(feature_maps):
    """Per-level NCHW maps ``[bs, Ncam, C, H, W]`` -> ``(feat [bs, Ncam*sum(HW), C],
    spatial_shape [Ncam, L, 2], scale_start_index [Ncam, L])``, camera-major, levels in order."""
    fms = [np.asarray(f, dtype=f32) for f in feature_maps]
    bs, nc, C = fms[0].shape[:3]
    shapes = [f.shape[3:5] for f in fms]
    per_cam = [f.reshape(bs, nc, C, -1) for f in fms]
    col = np.concatenate(per_cam, axis=-1).transpose(0, 1, 3, 2).reshape(bs, -1, C)
    hw = np.array([h * w for h, w in shapes], dtype=np.int64)
    starts_l = np.concatenate([[0], np.cumsum(hw)[:-1]])
    total = hw.sum()
    spatial = np.tile(np.array(shapes, dtype=np.int32)[None], (nc, 1, 1))
    start = (np.arange(nc)[:, None] * total + starts_l[None]).astype(np.int32)
    return np.ascontiguousarray(col), spatial, start


def deformable_aggregation(feat, spatial_shape, scale_start_index, uv_bacp2, weights, logits=True,
                           cam_range=None):
    """Operator semantics: ``out[b, a, g*D + d] = sum_{c, l, p} w[b,a,c,l,p,g] *
    bilinear(feat[b, cam c, level l], uv[b,a,c,p])[g*D + d]``, with ``w`` the softmax over
    (c, l, p) of the logits of group ``g`` (over all cameras, also when ``cam_range``
    restricts the cameras that are sampled).

    ``feat [bs, NF, C]``; ``uv_bacp2 [bs, A, Ncam, P, 2]``; ``weights [bs, A, Ncam, L, P, G]``.
    Bilinear sampling is ``grid_sample`` with zeros padding and align_corners=False at grid
    coordinate ``2u - 1`` (``test/dfa_pcc.py:339-344``)."""
    feat = np.asarray(feat, dtype=f32)
    bs, A, nc, npt = uv_bacp2.shape[:4]
    nl = spatial_shape.shape[1]
    G = weights.shape[-1]
    C = feat.shape[-1]
    D = C // G
    w = weights.astype(f32)
    if logits:
        flat = w.reshape(bs, A, -1, G)
        m = flat.max(axis=2, keepdims=True)
        e = np.exp(flat - m)
        w = (e / e.sum(axis=2, keepdims=True)).reshape(w.shape).astype(f32)
    out = np.zeros((bs, A, C), dtype=f32)
    cams = range(nc) if cam_range is None else range(cam_range[0], cam_range[1])
    for c in cams:
        for l in range(nl):
            Hh, Ww = int(spatial_shape[c, l, 0]), int(spatial_shape[c, l, 1])
            base = int(scale_start_index[c, l])
            gx = uv_bacp2[:, :, c, :, 0].astype(f32) * f32(2) - f32(1)  # [bs, A, P]
            gy = uv_bacp2[:, :, c, :, 1].astype(f32) * f32(2) - f32(1)
            ix = ((gx + f32(1)) * f32(Ww) - f32(1)) / f32(2)
            iy = ((gy + f32(1)) * f32(Hh) - f32(1)) / f32(2)
            with np.errstate(invalid="ignore"):
                x0 = np.floor(ix)
                y0 = np.floor(iy)
            x1, y1 = x0 + 1, y0 + 1
            taps = [
                (x0, y0, (x1 - ix) * (y1 - iy)),
                (x1, y0, (ix - x0) * (y1 - iy)),
                (x0, y1, (x1 - ix) * (iy - y0)),
                (x1, y1, (ix - x0) * (iy - y0)),
            ]
            sampled = np.zeros((bs, A, npt, C), dtype=f32)
            for tx, ty, tw in taps:
                with np.errstate(invalid="ignore"):
                    ok = (tx >= 0) & (tx < Ww) & (ty >= 0) & (ty < Hh)
                if not ok.any():
                    continue
                bi, ai, pi = np.nonzero(ok)
                pix = base + ty[ok].astype(np.int64) * Ww + tx[ok].astype(np.int64)
                vals = feat[bi, pix]  # [n, C]
                sampled[bi, ai, pi] += tw[ok].astype(f32)[:, None] * vals
            wl = w[:, :, c, l]  # [bs, A, P, G]
            contrib = sampled.reshape(bs, A, npt, G, D) * wl[..., None]
            out += contrib.sum(axis=2).reshape(bs, A, C)
    return out
