"""The C-ABI library: it loads, exports every function that include/s4d_dfa.h declares, and
rejects bad arguments on the host with a status code (no GPU needed: none of these calls
reaches a launch)."""
import ctypes as C
import os
import re

import pytest

from sparse4d_tt_b200 import _lib as L

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(REPO, "include", "s4d_dfa.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(s4d_[a-z_0-9]+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    if not os.path.exists(L.LIB_PATH):
        import importlib.util

        spec = importlib.util.spec_from_file_location("s4d_build", os.path.join(REPO, "sparse4d-tt_b200", "build.py"))
        b = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(b)
        b.build()
    return L.lib()


def test_every_declared_symbol_is_exported(lib):
    names = declared_functions()
    assert len(names) == 31, names
    for n in names:
        assert hasattr(lib, n), n
        assert n in L.SIGNATURES, f"{n} has no ctypes signature"


def test_no_extra_exports(lib):
    """Hidden visibility: only the declared API is exported."""
    import subprocess

    out = subprocess.run(["nm", "-D", "--defined-only", L.LIB_PATH], capture_output=True, text=True).stdout
    exported = {ln.split()[-1] for ln in out.splitlines() if " T " in ln}
    assert {n for n in exported if n.startswith("s4d_")} == set(declared_functions())


def test_status_strings_and_version(lib):
    assert L.status_string(0) == "S4D_OK"
    assert L.status_string(2) == "S4D_ERR_UNSUPPORTED_SHAPE"
    assert L.status_string(99) == "S4D_ERR_UNKNOWN"
    assert lib.s4d_abi_version() == 109 == L.ABI_VERSION


def test_dfa_workspace_bytes(lib):
    assert lib.s4d_dfa_workspace_bytes(2, 6, 4, 13, 8, 1) == 2 * 7 * 416 * 4 + 16
    assert lib.s4d_dfa_workspace_bytes(2, 6, 4, 13, 8, 0) == 0


def test_workspace_bytes(lib):
    assert lib.s4d_kps_workspace_bytes(1, 900, 6, 13) >= 4 * 69 + 4 * 69 * 32
    assert lib.s4d_kps_workspace_bytes(0, 900, 6, 13) == 0
    assert lib.s4d_kps_workspace_bytes(2, 900, 6, 13) > lib.s4d_kps_workspace_bytes(1, 900, 6, 13)


def _gather(lib, **kw):
    args = dict(feat=8, dtype=1, num_feat=100, shape=8, start=8, loc=8, w=8, wc=None, logits=1, layout=0, bs=1,
                A=4, nc=6, nl=4, np=13, G=8, C=256, cb=0, ce=6, out=8, flag=None)
    args.update(kw)
    st = lib.s4d_deformable_aggregation(
        args["feat"], args["dtype"], args["num_feat"], args["shape"], args["start"], args["loc"], args["w"],
        args["wc"], args["logits"], args["layout"], args["bs"], args["A"], args["nc"], args["nl"], args["np"],
        args["G"], args["C"], args["cb"], args["ce"], args["out"], args["flag"], args.get("ws"), args.get("wsb", 0),
        None)
    return st, lib.s4d_last_error().decode()


@pytest.mark.parametrize("kw,status,text", [
    (dict(C=128), L.S4D_ERR_UNSUPPORTED_SHAPE, "embed_dims"),
    (dict(G=3), L.S4D_ERR_UNSUPPORTED_SHAPE, "num_groups"),
    (dict(G=64), L.S4D_ERR_UNSUPPORTED_SHAPE, "num_groups"),
    (dict(np=200, nl=4), L.S4D_ERR_UNSUPPORTED_SHAPE, "12288"),
    (dict(dtype=7), L.S4D_ERR_INVALID_ARG, "feat_dtype"),
    (dict(layout=2), L.S4D_ERR_INVALID_ARG, "layout"),
    (dict(cb=4, ce=2), L.S4D_ERR_INVALID_ARG, "cam_begin"),
    (dict(ce=7), L.S4D_ERR_INVALID_ARG, "cam_begin"),
    (dict(wc=8, layout=1), L.S4D_ERR_INVALID_ARG, "weights_cam"),
    (dict(wc=8, logits=0), L.S4D_ERR_INVALID_ARG, "split"),
    (dict(feat=None), L.S4D_ERR_INVALID_ARG, "null"),
    (dict(feat=24), L.S4D_ERR_INVALID_ARG, "16-byte"),
    (dict(bs=-1), L.S4D_ERR_INVALID_ARG, "positive"),
    (dict(feat=16, wc=16, ws=24, wsb=1 << 20), L.S4D_ERR_INVALID_ARG, "workspace"),
    (dict(feat=16, wc=16, ws=16, wsb=64), L.S4D_ERR_INVALID_ARG, "workspace"),
])
def test_gather_rejects_on_host(lib, kw, status, text):
    st, msg = _gather(lib, **kw)
    assert st == status, (st, msg)
    assert text in msg


def test_gather_empty_batch_is_a_noop(lib):
    st, msg = _gather(lib, bs=0, feat=None, out=None)
    assert st == L.S4D_OK, msg


def _kps(lib, **kw):
    a = dict(anchor=16, adim=11, fix=16, nfix=7, learn=16, nlearn=6, proj=16, wh=16, bs=1, A=4, nc=6, layout=0,
             kp=None, loc=16, mask=None, idx=16, cnt=16, ws=16, wsb=1 << 20)
    a.update(kw)
    st = lib.s4d_kps_project(a["anchor"], a["adim"], a["fix"], a["nfix"], a["learn"], a["nlearn"], a["proj"],
                             a["wh"], a["bs"], a["A"], a["nc"], a["layout"], a["kp"], a["loc"], a["mask"], a["idx"],
                             a["cnt"], a["ws"], a["wsb"], None)
    return st, lib.s4d_last_error().decode()


@pytest.mark.parametrize("kw,status,text", [
    (dict(adim=7), L.S4D_ERR_INVALID_ARG, "anchor_dim"),
    (dict(layout=5), L.S4D_ERR_INVALID_ARG, "layout"),
    (dict(nfix=-1), L.S4D_ERR_INVALID_ARG, "negative"),
    (dict(anchor=None), L.S4D_ERR_INVALID_ARG, "null"),
    (dict(learn=None), L.S4D_ERR_INVALID_ARG, "learnable"),
    (dict(idx=20), L.S4D_ERR_INVALID_ARG, "visible_idx"),
    (dict(loc=20), L.S4D_ERR_INVALID_ARG, "sample_location"),
    (dict(ws=None), L.S4D_ERR_INVALID_ARG, "workspace"),
    (dict(wsb=8), L.S4D_ERR_INVALID_ARG, "workspace"),
    (dict(A=1 << 30), L.S4D_ERR_UNSUPPORTED_SHAPE, "2^31"),
    (dict(nfix=0, nlearn=0), L.S4D_ERR_INVALID_ARG, "keypoints"),
])
def test_kps_rejects_on_host(lib, kw, status, text):
    st, msg = _kps(lib, **kw)
    assert st == status, (st, msg)
    assert text in msg


def test_kps_fused_rejects_on_host(lib):
    st = lib.s4d_kps_project_fused(16, 16, 5, 16, 16, 4, 6, 13, 16, None)
    assert st == L.S4D_ERR_INVALID_ARG
    st = lib.s4d_kps_project_fused(None, 16, 11, 16, 16, 4, 6, 13, 16, None)
    assert st == L.S4D_ERR_INVALID_ARG
    st = lib.s4d_kps_project_fused(16, 16, 11, 16, 16, 0, 6, 13, 16, None)
    assert st == L.S4D_OK  # nothing to do


def test_last_error_is_per_thread(lib):
    import threading

    st, msg = _gather(lib, C=128)
    assert "embed_dims" in msg
    seen = {}

    def other():
        seen["msg"] = lib.s4d_last_error().decode()

    t = threading.Thread(target=other)
    t.start()
    t.join()
    assert seen["msg"] == ""
    assert "embed_dims" in lib.s4d_last_error().decode()


def test_ops_reject_cpu_tensors():
    """No CPU fallback: the operators refuse host tensors."""
    import torch

    from sparse4d_tt_b200 import ops

    feat = torch.zeros(1, 10, 256)
    shape = torch.zeros(6, 4, 2, dtype=torch.int32)
    start = torch.zeros(6, 4, dtype=torch.int32)
    loc = torch.zeros(1, 2, 6, 13, 2)
    w = torch.zeros(1, 2, 6, 4, 13, 8)
    with pytest.raises(ValueError, match="CUDA"):
        ops.deformable_aggregation_into(torch.zeros(1, 2, 256), feat, shape, start, loc, w)
    with pytest.raises(ValueError, match="CUDA"):
        ops.kps_project_into(torch.zeros(1, 2, 11), torch.zeros(1, 2, 18), torch.zeros(7, 3),
                             torch.zeros(1, 6, 4, 4), torch.zeros(1, 6, 2))


def _wfc(lib, **kw):
    a = dict(inst=16, ild=256, emb=16, eld=256, rows=900, wfc=16, wkps=16, n=416, m=18, C=256, bias=16, logits=16,
             learn=16)
    a.update(kw)
    st = lib.s4d_dfa_weights_fc(a["inst"], a["ild"], a["emb"], a["eld"], a["rows"], a["wfc"], a["wkps"], a["bias"],
                                a["n"], a["m"], a["C"], a["logits"], a["learn"], None, None)
    return st, lib.s4d_last_error().decode()


def _oproj(lib, **kw):
    a = dict(feat=16, rows=900, w=16, b=16, inst=16, ild=512, mode=2, out=16, old=512, C=256)
    a.update(kw)
    st = lib.s4d_dfa_output_proj(a["feat"], a["rows"], a["w"], a["b"], a["inst"], a["ild"], a["mode"], a["out"],
                                 a["old"], a["C"], None, None)
    return st, lib.s4d_last_error().decode()


@pytest.mark.parametrize("kw,status,text", [
    (dict(C=128), L.S4D_ERR_UNSUPPORTED_SHAPE, "embed_dims"),
    (dict(m=40), L.S4D_ERR_UNSUPPORTED_SHAPE, "num_learnable <= 32"),
    (dict(n=408), L.S4D_ERR_UNSUPPORTED_SHAPE, "num_logits 416"),
    (dict(rows=-1), L.S4D_ERR_INVALID_ARG, "sizes"),
    (dict(inst=None), L.S4D_ERR_INVALID_ARG, "null"),
    (dict(learn=None), L.S4D_ERR_INVALID_ARG, "null"),
    (dict(wkps=None), L.S4D_ERR_INVALID_ARG, "null"),
    (dict(wkps=8), L.S4D_ERR_INVALID_ARG, "misaligned"),
    (dict(ild=254), L.S4D_ERR_INVALID_ARG, "strides"),
    (dict(eld=258), L.S4D_ERR_INVALID_ARG, "strides"),
    (dict(inst=8), L.S4D_ERR_INVALID_ARG, "misaligned"),
    (dict(logits=20), L.S4D_ERR_INVALID_ARG, "misaligned"),
])
def test_weights_fc_rejects(lib, kw, status, text):
    st, msg = _wfc(lib, **kw)
    assert st == status and text in msg, msg


def test_weights_fc_zero_rows_is_ok(lib):
    assert _wfc(lib, rows=0)[0] == L.S4D_OK


@pytest.mark.parametrize("kw,status,text", [
    (dict(C=512), L.S4D_ERR_UNSUPPORTED_SHAPE, "embed_dims"),
    (dict(mode=3), L.S4D_ERR_INVALID_ARG, "residual_mode"),
    (dict(old=256), L.S4D_ERR_INVALID_ARG, "out_ld"),
    (dict(old=514), L.S4D_ERR_INVALID_ARG, "out_ld"),
    (dict(ild=100), L.S4D_ERR_INVALID_ARG, "instance_ld"),
    (dict(inst=None), L.S4D_ERR_INVALID_ARG, "null"),
    (dict(b=8), L.S4D_ERR_INVALID_ARG, "misaligned"),
    (dict(out=8), L.S4D_ERR_INVALID_ARG, "misaligned"),
])
def test_output_proj_rejects(lib, kw, status, text):
    st, msg = _oproj(lib, **kw)
    assert st == status and text in msg, msg


def test_output_proj_modes_without_residual(lib):
    assert _oproj(lib, rows=0, inst=None, mode=0, old=256)[0] == L.S4D_OK


def _cam(lib, **kw):
    a = dict(proj=16, bs=32, nc=6, w=16, n=416, C=256, emb=None, out=16, ws=16, wsb=32 * 6 * 256 * 4)
    a.update(kw)
    w = a["w"]
    st = lib.s4d_dfa_camera_logits(a["proj"], a["bs"], a["nc"], w, w, w, w, w, w, w, w, w, w, a["n"], a["C"], a["emb"],
                                   a["out"], a["ws"], a["wsb"], None)
    return st, lib.s4d_last_error().decode()


@pytest.mark.parametrize("kw,status,text", [
    (dict(nc=9), L.S4D_ERR_UNSUPPORTED_SHAPE, "1..8 cameras"),
    (dict(C=128), L.S4D_ERR_UNSUPPORTED_SHAPE, "embed_dims 256"),
    (dict(nc=0), L.S4D_ERR_INVALID_ARG, "bad sizes"),
    (dict(bs=-1), L.S4D_ERR_INVALID_ARG, "bad sizes"),
    (dict(out=None), L.S4D_ERR_INVALID_ARG, "null"),
    (dict(w=8), L.S4D_ERR_INVALID_ARG, "16-byte aligned"),
    (dict(ws=None), L.S4D_ERR_INVALID_ARG, "workspace"),
    (dict(wsb=1000), L.S4D_ERR_INVALID_ARG, "workspace"),
])
def test_camera_logits_rejects(lib, kw, status, text):
    st, msg = _cam(lib, **kw)
    assert st == status and text in msg, msg


def test_camera_logits_zero_frames_is_ok(lib):
    assert _cam(lib, bs=0)[0] == L.S4D_OK


def test_camera_workspace_bytes(lib):
    assert lib.s4d_dfa_camera_workspace_bytes(32, 6, 256) == 32 * 6 * 256 * 4
    assert lib.s4d_dfa_camera_workspace_bytes(0, 6, 256) == 0


def _terms(lib, **kw):
    a = dict(proj=16, bs=32, nc=6, w=16, n=416, C=256, emb=None, out=16, ws=16,
             wsb=lib.s4d_dfa_workspace_bytes(32, 6, 4, 13, 8, 1))
    a.update(kw)
    w = a["w"]
    st = lib.s4d_dfa_camera_terms(a["proj"], a["bs"], a["nc"], w, w, w, w, w, w, w, w, w, w, a["n"], a["C"], a["emb"],
                                  a["out"], a["ws"], a["wsb"], None)
    return st, lib.s4d_last_error().decode()


@pytest.mark.parametrize("kw,status,text", [
    (dict(nc=9), L.S4D_ERR_UNSUPPORTED_SHAPE, "1..8 cameras"),
    (dict(C=128), L.S4D_ERR_UNSUPPORTED_SHAPE, "embed_dims 256"),
    (dict(n=520), L.S4D_ERR_UNSUPPORTED_SHAPE, "512 logits"),
    (dict(n=412), L.S4D_ERR_UNSUPPORTED_SHAPE, "8 groups"),
    (dict(nc=0), L.S4D_ERR_INVALID_ARG, "bad sizes"),
    (dict(bs=-1), L.S4D_ERR_INVALID_ARG, "bad sizes"),
    (dict(out=None), L.S4D_ERR_INVALID_ARG, "null"),
    (dict(w=8), L.S4D_ERR_INVALID_ARG, "16-byte aligned"),
    (dict(ws=8), L.S4D_ERR_INVALID_ARG, "workspace"),
    (dict(wsb=1000), L.S4D_ERR_INVALID_ARG, "workspace"),
])
def test_camera_terms_rejects_on_host(lib, kw, status, text):
    """Every argument check of the one-launch camera terms runs before a launch (no GPU here)."""
    st, msg = _terms(lib, **kw)
    assert st == status and text in msg, msg


def test_camera_terms_zero_frames_is_ok(lib):
    assert _terms(lib, bs=0)[0] == L.S4D_OK
    assert _terms(lib, bs=0, ws=None, n=412)[0] == L.S4D_OK


def _pack(lib, **kw):
    a = dict(levels=[16, 16], layout=0, sd=0, bs=2, nc=6, nl=2, hw=[4, 4, 2, 2], C=256, dd=1, out=16)
    a.update(kw)
    lv = None if a["levels"] is None else (C.c_void_p * len(a["levels"]))(*a["levels"])
    hw = (C.c_int32 * len(a["hw"]))(*a["hw"])
    st = lib.s4d_pack_feature_maps(lv, a["layout"], a["sd"], a["bs"], a["nc"], a["nl"], hw, a["C"], a["dd"], a["out"],
                                   None)
    return st, lib.s4d_last_error().decode()


@pytest.mark.parametrize("kw,status,text", [
    (dict(layout=2), L.S4D_ERR_INVALID_ARG, "layout"),
    (dict(sd=5), L.S4D_ERR_INVALID_ARG, "dtype"),
    (dict(C=96), L.S4D_ERR_UNSUPPORTED_SHAPE, "multiple of 64"),
    (dict(nl=9, levels=[16] * 9, hw=[2] * 18), L.S4D_ERR_UNSUPPORTED_SHAPE, "8 levels"),
    (dict(levels=[16, 8]), L.S4D_ERR_INVALID_ARG, "misaligned"),
    (dict(hw=[4, 0, 2, 2]), L.S4D_ERR_INVALID_ARG, "positive"),
    (dict(out=None), L.S4D_ERR_INVALID_ARG, "null"),
    (dict(out=8), L.S4D_ERR_INVALID_ARG, "16-byte aligned"),
])
def test_pack_rejects(lib, kw, status, text):
    st, msg = _pack(lib, **kw)
    assert st == status and text in msg, msg


def test_pack_zero_batch_is_ok(lib):
    assert _pack(lib, bs=0)[0] == L.S4D_OK


def test_instance_bank_rejects(lib):
    assert lib.s4d_instance_bank_project(16, 16, None, -1, 10, 16, None) == L.S4D_ERR_INVALID_ARG
    assert lib.s4d_instance_bank_project(None, 16, None, 1, 10, 16, None) == L.S4D_ERR_INVALID_ARG
    assert lib.s4d_instance_bank_project(16, 16, None, 0, 10, 16, None) == L.S4D_OK
    args = [16, 16, 16, None, 0.6, 2, 900, 10, 256, 600, 16, 16, None, None, None]
    assert lib.s4d_instance_bank_cache(*args[:9], 901, *args[10:]) == L.S4D_ERR_INVALID_ARG  # num_temp > A
    assert lib.s4d_instance_bank_cache(*args[:6], 5000, *args[7:]) == L.S4D_ERR_UNSUPPORTED_SHAPE
    assert lib.s4d_instance_bank_cache(None, *args[1:]) == L.S4D_ERR_INVALID_ARG
    uargs = [16, 16, 16, 16, 16, None, 2, 900, 10, 256, 600, 16, 16, None, None]
    assert lib.s4d_instance_bank_update(*uargs[:11], None, *uargs[12:]) == L.S4D_ERR_INVALID_ARG
    assert lib.s4d_instance_bank_update(*uargs[:6], 0, *uargs[7:]) == L.S4D_OK


def test_prepared_factors_rejects(lib):
    st, msg = _gather(lib, logits=2, wc=8)  # no workspace
    assert st == L.S4D_ERR_INVALID_ARG and "prepared" in msg
    st, msg = _gather(lib, logits=2, wc=None, ws=16, wsb=1 << 20)
    assert st == L.S4D_ERR_INVALID_ARG and "prepared" in msg
    st, msg = _gather(lib, logits=3)
    assert st == L.S4D_ERR_INVALID_ARG and "0, 1 or 2" in msg
    assert lib.s4d_dfa_camera_factors(16, 2, 6, 4, 13, 8, 16, 16, None) == L.S4D_ERR_INVALID_ARG  # too small
    assert lib.s4d_dfa_camera_factors(16, 0, 6, 4, 13, 8, None, 0, None) == L.S4D_OK


def _gather_anchors(lib, **kw):
    a = dict(feat=16, dtype=1, num_feat=100, shape=16, start=16, anchor=16, adim=11, fix=16, nfix=7, learn=16,
             proj=16, wh=16, w=16, wc=16, bs=1, A=4, nc=6, nl=4, np=13, G=8, C=256, cb=0, ce=6, out=16, flag=None,
             ws=16, wsb=1 << 20)
    a.update(kw)
    st = lib.s4d_deformable_aggregation_anchors(
        a["feat"], a["dtype"], a["num_feat"], a["shape"], a["start"], a["anchor"], a["adim"], a["fix"], a["nfix"],
        a["learn"], a["proj"], a["wh"], a["w"], a["wc"], a["bs"], a["A"], a["nc"], a["nl"], a["np"], a["G"], a["C"],
        a["cb"], a["ce"], a["out"], a["flag"], a["ws"], a["wsb"], None)
    return st, lib.s4d_last_error().decode()


@pytest.mark.parametrize("kw,status,text", [
    (dict(nc=5, ce=5), L.S4D_ERR_UNSUPPORTED_SHAPE, "6 cameras"),
    (dict(np=12), L.S4D_ERR_UNSUPPORTED_SHAPE, "13 points"),
    (dict(adim=7), L.S4D_ERR_INVALID_ARG, "anchor_dim"),
    (dict(nfix=14), L.S4D_ERR_INVALID_ARG, "num_fix"),
    (dict(anchor=None), L.S4D_ERR_INVALID_ARG, "null"),
    (dict(learn=None), L.S4D_ERR_INVALID_ARG, "null"),
    (dict(proj=8), L.S4D_ERR_INVALID_ARG, "projection_mat"),
    (dict(wh=4), L.S4D_ERR_INVALID_ARG, "image_wh"),
    (dict(w=8), L.S4D_ERR_INVALID_ARG, "weights"),
    (dict(ws=None, wsb=0), L.S4D_ERR_INVALID_ARG, "prepared"),
    (dict(wc=None), L.S4D_ERR_INVALID_ARG, "prepared"),
    (dict(C=128), L.S4D_ERR_UNSUPPORTED_SHAPE, "embed_dims"),
    (dict(wsb=64), L.S4D_ERR_INVALID_ARG, "workspace"),
])
def test_gather_anchors_rejects_on_host(lib, kw, status, text):
    st, msg = _gather_anchors(lib, **kw)
    assert st == status, (st, msg)
    assert text in msg


def test_gather_anchors_empty_batch_is_a_noop(lib):
    st, msg = _gather_anchors(lib, bs=0, anchor=None, learn=None, feat=None, out=None)
    assert st == L.S4D_OK, msg


def test_size_products_that_overflow_int64_are_rejected(lib):
    """Sizes whose product overflows int64 must be rejected, not wrapped to a small value that
    passes the limits (every check below returns before any pointer is used)."""
    big = 1 << 40
    st, msg = _kps(lib, bs=big, A=big)
    assert st == L.S4D_ERR_UNSUPPORTED_SHAPE and "2^31" in msg, msg
    st, msg = _kps(lib, bs=1 << 33, A=1 << 31)  # product 2^64 wraps to 0 in int64
    assert st == L.S4D_ERR_UNSUPPORTED_SHAPE, msg
    assert lib.s4d_kps_workspace_bytes(big, big, 6, 13) == 0
    st, msg = _gather(lib, bs=1 << 33, A=1 << 31)
    assert st == L.S4D_ERR_UNSUPPORTED_SHAPE and "too many" in msg, msg
    st, msg = _gather(lib, np=1 << 40, nl=1 << 40)
    assert st == L.S4D_ERR_UNSUPPORTED_SHAPE and "12288" in msg, msg
    assert lib.s4d_kps_project_fused(16, 16, 11, 16, 16, 1 << 40, 1 << 30, 13, 16, None) == L.S4D_ERR_UNSUPPORTED_SHAPE
    assert lib.s4d_dfa_workspace_bytes(2, 1 << 40, 1 << 40, 13, 8, 1) == 0
    assert lib.s4d_dfa_camera_workspace_bytes(1 << 40, 1 << 40, 256) == 0
    assert lib.s4d_instance_bank_project(16, 16, None, 1 << 33, 1 << 31, 16, None) == L.S4D_ERR_UNSUPPORTED_SHAPE


def test_noalloc_limit_is_checked_on_the_host(lib):
    """s4d_kps_project_noalloc rejects bs*A*Ncam*P above its built-in scratch (4,194,304
    elements), including products that overflow, before touching the GPU."""
    def call(bs, A, nc, nfix, nlearn):
        st = lib.s4d_kps_project_noalloc(16, 11, 16, nfix, 16, nlearn, 16, 16, bs, A, nc, 0, None, None, None,
                                         None, None, None)
        return st, lib.s4d_last_error().decode()

    st, msg = call(1, 838861, 1, 5, 0)  # 4,194,305 elements
    assert st == L.S4D_ERR_UNSUPPORTED_SHAPE and "scratch limit" in msg, msg
    st, msg = call(1 << 33, 1 << 31, 1, 1, 0)  # wraps to 0 in int64
    assert st == L.S4D_ERR_UNSUPPORTED_SHAPE and "scratch limit" in msg, msg
    st, msg = call(1, 1, 1, 1 << 62, 1 << 62)
    assert st == L.S4D_ERR_UNSUPPORTED_SHAPE, msg


def test_tc_wait_limit_is_per_thread_and_restorable(lib):
    import threading

    prev = lib.s4d_set_tc_wait_limit_ns(12345)
    assert prev == 2_000_000_000
    seen = {}

    def other():
        seen["v"] = lib.s4d_set_tc_wait_limit_ns(7)

    t = threading.Thread(target=other)
    t.start()
    t.join()
    assert seen["v"] == 2_000_000_000  # another thread keeps its own default
    assert lib.s4d_set_tc_wait_limit_ns(prev) == 12345


def _oproj_sum(lib, **kw):
    a = dict(feat=16, feat2=16, total=1800, row0=900, rows=900, w=16, b=16, inst=16, ild=512, mode=2, out=16,
             old=512, C=256)
    a.update(kw)
    st = lib.s4d_dfa_output_proj_sum(a["feat"], a["feat2"], a["total"], a["row0"], a["rows"], a["w"], a["b"],
                                     a["inst"], a["ild"], a["mode"], a["out"], a["old"], a["C"], None, None)
    return st, lib.s4d_last_error().decode()


@pytest.mark.parametrize("kw,status,text", [
    (dict(row0=901), L.S4D_ERR_INVALID_ARG, "outside the sources"),
    (dict(row0=-1), L.S4D_ERR_INVALID_ARG, "negative"),
    (dict(rows=-1), L.S4D_ERR_INVALID_ARG, "negative"),
    (dict(total=1 << 31, row0=0), L.S4D_ERR_UNSUPPORTED_SHAPE, "feature_rows"),
    (dict(feat2=None), L.S4D_ERR_INVALID_ARG, "features2"),
    (dict(feat2=8), L.S4D_ERR_INVALID_ARG, "features2"),
    (dict(feat=8), L.S4D_ERR_INVALID_ARG, "s4d_dfa_output_proj_sum: misaligned"),
    (dict(C=512), L.S4D_ERR_UNSUPPORTED_SHAPE, "s4d_dfa_output_proj_sum: embed_dims"),
    (dict(old=256), L.S4D_ERR_INVALID_ARG, "out_ld"),
    (dict(mode=3), L.S4D_ERR_INVALID_ARG, "residual_mode"),
])
def test_output_proj_sum_rejects(lib, kw, status, text):
    st, msg = _oproj_sum(lib, **kw)
    assert st == status and text in msg, msg


def test_output_proj_sum_zero_rows_is_ok(lib):
    assert _oproj_sum(lib, rows=0, row0=1800, feat2=None)[0] == L.S4D_OK


def test_peer_entry_points_reject_on_host(lib):
    assert lib.s4d_ipc_handle_bytes() == 64
    slots = (C.c_void_p * 8)(16, 32)
    arr = C.cast(slots, C.c_void_p)
    for world, rank, text in ((0, 0, "world"), (9, 0, "world"), (2, 2, "rank"), (2, -1, "rank")):
        st = lib.s4d_peer_signal_wait(64, arr, rank, world, 1, 1000, None, None)
        assert st != L.S4D_OK and text in lib.s4d_last_error().decode()
    assert lib.s4d_peer_signal_wait(None, arr, 0, 2, 1, 1000, None, None) == L.S4D_ERR_INVALID_ARG
    assert lib.s4d_peer_signal_wait(64, None, 0, 2, 1, 1000, None, None) == L.S4D_ERR_INVALID_ARG
    assert lib.s4d_peer_signal_wait(66, arr, 0, 2, 1, 1000, None, None) == L.S4D_ERR_INVALID_ARG
    bad = (C.c_void_p * 8)(16, 0)  # rank 0's peer (rank 1) has no slots
    st = lib.s4d_peer_signal_wait(64, C.cast(bad, C.c_void_p), 0, 2, 1, 1000, None, None)
    assert st == L.S4D_ERR_INVALID_ARG and "peer slots" in lib.s4d_last_error().decode()
    # one rank alone has nobody to wait for: nothing is launched
    assert lib.s4d_peer_signal_wait(64, arr, 0, 1, 1, 1000, None, None) == L.S4D_OK
    off = C.c_uint64(0)
    handle = C.create_string_buffer(64)
    assert lib.s4d_ipc_export(None, handle, C.byref(off)) == L.S4D_ERR_INVALID_ARG
    base = C.c_void_p()
    assert lib.s4d_ipc_open(None, C.byref(base)) == L.S4D_ERR_INVALID_ARG
    assert lib.s4d_ipc_close(None) == L.S4D_ERR_INVALID_ARG
    # the device-epoch variant
    st = lib.s4d_peer_signal_wait_counter(64, arr, 0, 2, None, 1, 1000, None, None)
    assert st == L.S4D_ERR_INVALID_ARG and "epoch counter" in lib.s4d_last_error().decode()
    st = lib.s4d_peer_signal_wait_counter(64, arr, 0, 2, 66, 1, 1000, None, None)
    assert st == L.S4D_ERR_INVALID_ARG and "misaligned epoch counter" in lib.s4d_last_error().decode()
    st = lib.s4d_peer_signal_wait_counter(64, arr, 0, 2, 128, 2, 1000, None, None)
    assert st == L.S4D_ERR_INVALID_ARG and "advance" in lib.s4d_last_error().decode()
    st = lib.s4d_peer_signal_wait_counter(64, arr, 3, 2, 128, 1, 1000, None, None)
    assert st == L.S4D_ERR_INVALID_ARG and "s4d_peer_signal_wait_counter: rank" in lib.s4d_last_error().decode()
    # one rank, no advance: nothing to publish, wait for or count
    assert lib.s4d_peer_signal_wait_counter(64, arr, 0, 1, 128, 0, 1000, None, None) == L.S4D_OK


def test_gather_routing_rejects_on_host(lib):
    """s4d_deformable_aggregation_anchors_peer: the routed row range and out_peer are checked
    before anything launches."""
    def call(out_peer, begin, end, out=16):
        return lib.s4d_deformable_aggregation_anchors_peer(
            16, 1, 100, 16, 16, 16, 11, 16, 7, 16, 16, 16, 16, 16, 2, 900, 6, 4, 13, 8, 256, 0, 6, out, out_peer,
            begin, end, None, 64, 1 << 20, None), lib.s4d_last_error().decode()
    for begin, end in ((-1, 5), (10, 5), (0, 1801)):
        st, msg = call(32, begin, end)
        assert st == L.S4D_ERR_INVALID_ARG and "peer_row_begin" in msg, msg
    st, msg = call(None, 900, 1800)
    assert st == L.S4D_ERR_INVALID_ARG and "out_peer" in msg, msg
    st, msg = call(40, 900, 1800)
    assert st == L.S4D_ERR_INVALID_ARG and "out_peer" in msg, msg
    st, msg = call(32, 900, 1800, out=20)
    assert st == L.S4D_ERR_INVALID_ARG and "16-byte" in msg, msg


def test_layer_norm_rejects_on_host(lib):
    def call(x=16, w=16, b=16, y=32, rows=10, width=256, eps=1e-5):
        return lib.s4d_layer_norm(x, w, b, y, rows, width, eps, None), lib.s4d_last_error().decode()
    for kw, status, text in ((dict(width=48), L.S4D_ERR_UNSUPPORTED_SHAPE, "width"),
                             (dict(rows=-1), L.S4D_ERR_INVALID_ARG, "negative"),
                             (dict(eps=-1.0), L.S4D_ERR_INVALID_ARG, "eps"),
                             (dict(x=None), L.S4D_ERR_INVALID_ARG, "null"),
                             (dict(w=None), L.S4D_ERR_INVALID_ARG, "bias needs a weight"),
                             (dict(y=18), L.S4D_ERR_INVALID_ARG, "misaligned"),
                             (dict(rows=1 << 40), L.S4D_ERR_UNSUPPORTED_SHAPE, "too many")):
        st, msg = call(**kw)
        assert st == status and text in msg, (kw, msg)
    assert call(rows=0)[0] == L.S4D_OK
