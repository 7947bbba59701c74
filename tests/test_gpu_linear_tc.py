"""The tensor-core (tcgen05, TF32) linears around the gather against float64 references.

TF32 keeps 10 mantissa bits of each operand, so one product a*w carries a relative error below
2^-9 and the fp32 accumulation of K <= 512 terms adds less than 2^-14 of sum|a||w|.  Each
output is checked against the rigorous bound 2^-8 * sum_k |a_k||w_k| (float64), and the median
error against a much tighter 2^-12 of the same scale so that a systematic slip cannot hide
inside the bound."""
import pytest
import torch

from sparse4d_tt_b200 import ops

pytestmark = pytest.mark.gpu

BOUND = 2.0 ** -8
TYPICAL = 2.0 ** -12


def _check(got, ref, scale, what):
    err = (got.double() - ref).abs()
    worst = (err / scale.clamp_min(1e-30)).max().item()
    typical = (err / scale.clamp_min(1e-30)).median().item()
    print(f"{what}: max err/bound-scale {worst:.3e}, median {typical:.3e}")
    assert worst <= BOUND, what
    assert typical <= TYPICAL, what


def _weights(n, m, c, gen, dev):
    w_fc = (torch.rand(n, c, generator=gen) * 2 - 1) * (6 / (n + c)) ** 0.5
    w_kps = (torch.rand(m, c, generator=gen) * 2 - 1) * (6 / (m + c)) ** 0.5
    b_kps = torch.randn(m, generator=gen)
    return w_fc.to(dev), w_kps.to(dev), b_kps.to(dev)


@pytest.mark.parametrize("rows", [1, 4, 127, 128, 129, 900, 1800, 7200, 18945, 20000, 28800])
def test_weights_fc_matches_float64(cuda_device, rows):
    """Column groups for few row tiles, whole tiles per CTA otherwise, up to the two waves of
    tiles of the 32-frame layer (28,800 rows)."""
    dev = torch.device("cuda:0")
    gen = torch.Generator().manual_seed(rows)
    n, m, c = 416, 18, 256
    w_fc, w_kps, b_kps = _weights(n, m, c, gen, dev)
    inst = torch.randn(rows, c, generator=gen).to(dev)
    embed = torch.randn(rows, c, generator=gen).to(dev)
    logits = torch.full((rows, n), float("nan"), device=dev)
    learn = torch.full((rows, m), float("nan"), device=dev)
    flag = torch.zeros(1, dtype=torch.int32, device=dev)
    ops.weights_fc_into(logits, learn, inst, embed, w_fc, w_kps, b_kps, error_flag=flag)
    torch.cuda.synchronize()
    assert flag.item() == 0
    i64, e64, wf, wk = inst.double(), embed.double(), w_fc.double(), w_kps.double()
    _check(logits, (i64 + e64) @ wf.T, (i64.abs() + e64.abs()) @ wf.abs().T, f"logits rows={rows}")
    _check(learn, i64 @ wk.T + b_kps.double(), i64.abs() @ wk.abs().T + 1e-6, f"learnable rows={rows}")


def test_weights_fc_reads_strided_rows(cuda_device):
    """The layer feeds the previous layer's [rows, 2C] output as the instance feature: a row
    stride of 512 floats, read in place by TMA."""
    dev = torch.device("cuda:0")
    gen = torch.Generator().manual_seed(7)
    rows, n, m, c = 1000, 416, 18, 256
    w_fc, w_kps, b_kps = _weights(n, m, c, gen, dev)
    wide = torch.randn(rows, 2 * c, generator=gen).to(dev)
    inst = wide[:, :c]
    embed_wide = torch.randn(rows, 3 * c, generator=gen).to(dev)
    embed = embed_wide[:, c:2 * c]
    assert ops.row_view(inst, c).stride(0) == 2 * c and ops.row_view(embed, c).stride(0) == 3 * c
    logits = torch.empty(rows, n, device=dev)
    learn = torch.empty(rows, m, device=dev)
    ops.weights_fc_into(logits, learn, ops.row_view(inst, c), ops.row_view(embed, c), w_fc, w_kps, b_kps)
    ref_l = torch.empty_like(logits)
    ref_k = torch.empty_like(learn)
    ops.weights_fc_into(ref_l, ref_k, inst.contiguous(), embed.contiguous(), w_fc, w_kps, b_kps)
    torch.cuda.synchronize()
    assert torch.equal(logits, ref_l) and torch.equal(learn, ref_k)


@pytest.mark.parametrize("m", [0, 1, 18, 32])
def test_weights_fc_learnable_widths(cuda_device, m):
    """No learnable part, and up to the 32 columns of the learnable MMA."""
    dev = torch.device("cuda:0")
    gen = torch.Generator().manual_seed(30 + m)
    rows, n, c = 333, 416, 256
    w_fc, w_kps, b_kps = _weights(n, max(m, 1), c, gen, dev)
    inst = torch.randn(rows, c, generator=gen).to(dev)
    embed = torch.randn(rows, c, generator=gen).to(dev)
    logits = torch.empty(rows, n, device=dev)
    learn = torch.full((rows, m), float("nan"), device=dev) if m else None
    ops.weights_fc_into(logits, learn, inst, embed, w_fc, w_kps[:m].contiguous() if m else None,
                        b_kps[:m].contiguous() if m else None)
    torch.cuda.synchronize()
    i64, e64, wf = inst.double(), embed.double(), w_fc.double()
    _check(logits, (i64 + e64) @ wf.T, (i64.abs() + e64.abs()) @ wf.abs().T, f"logits m={m}")
    if m:
        wk = w_kps[:m].double()
        _check(learn, i64 @ wk.T + b_kps[:m].double(), i64.abs() @ wk.abs().T + 1e-6, f"learnable m={m}")


@pytest.mark.parametrize("mode", ["cat", "add", "none"])
@pytest.mark.parametrize("rows", [1, 129, 900, 7200, 28800])
def test_output_proj_residual_modes(cuda_device, mode, rows):
    dev = torch.device("cuda:0")
    gen = torch.Generator().manual_seed(rows + len(mode))
    c = 256
    w = ((torch.rand(c, c, generator=gen) * 2 - 1) * (3 / c) ** 0.5).to(dev)
    b = torch.randn(c, generator=gen).to(dev)
    feats = torch.randn(rows, c, generator=gen).to(dev)
    inst_wide = torch.randn(rows, 2 * c, generator=gen).to(dev)
    inst = inst_wide[:, :c]  # strided, as in a stacked decoder
    width = 2 * c if mode == "cat" else c + 8  # "add"/"none": 8 spare columns must stay untouched
    out = torch.full((rows, width), -7.0, device=dev)
    flag = torch.zeros(1, dtype=torch.int32, device=dev)
    ops.output_proj_into(out, feats, w, b, None if mode == "none" else inst, mode, error_flag=flag)
    torch.cuda.synchronize()
    assert flag.item() == 0
    f64, w64 = feats.double(), w.double()
    ref = f64 @ w64.T + b.double()
    scale = f64.abs() @ w64.abs().T + 1e-6
    if mode == "add":
        ref = ref + inst.double()
    _check(out[:, :c], ref, scale, f"output_proj {mode} rows={rows}")
    if mode == "cat":
        assert torch.equal(out[:, c:], inst)
    else:
        assert torch.all(out[:, c:] == -7.0)


def test_linear_tc_zero_rows(cuda_device):
    dev = torch.device("cuda:0")
    c = 256
    w = torch.randn(c, c, device=dev)
    out = torch.empty(0, 2 * c, device=dev)
    ops.output_proj_into(out, torch.empty(0, c, device=dev), w, None, torch.empty(0, c, device=dev), "cat")
    ops.weights_fc_into(torch.empty(0, 416, device=dev), torch.empty(0, 18, device=dev), torch.empty(0, c, device=dev),
                        torch.empty(0, c, device=dev), torch.randn(416, c, device=dev), torch.randn(18, c, device=dev))
    torch.cuda.synchronize()


def test_linear_tc_in_cuda_graph(cuda_device):
    """Both kernels capture into a CUDA graph and replay with new inputs."""
    dev = torch.device("cuda:0")
    gen = torch.Generator().manual_seed(11)
    rows, c = 900, 256
    w_fc, w_kps, b_kps = _weights(416, 18, c, gen, dev)
    w = torch.randn(c, c, generator=gen).to(dev) * 0.05
    b = torch.randn(c, generator=gen).to(dev)
    inst = torch.randn(rows, c, generator=gen).to(dev)
    embed = torch.randn(rows, c, generator=gen).to(dev)
    logits, learn = torch.empty(rows, 416, device=dev), torch.empty(rows, 18, device=dev)
    out = torch.empty(rows, 2 * c, device=dev)

    def body():
        ops.weights_fc_into(logits, learn, inst, embed, w_fc, w_kps, b_kps)
        ops.output_proj_into(out, logits[:, :c].contiguous(), w, b, inst, "cat")

    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        body()
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        body()
    inst.copy_(torch.randn(rows, c, generator=gen).to(dev))
    g.replay()
    torch.cuda.synchronize()
    got_l, got_o = logits.clone(), out.clone()
    body()
    torch.cuda.synchronize()
    assert torch.equal(got_l, logits) and torch.equal(got_o, out)


def test_wait_timeout_sets_flag_and_next_launch_is_clean(cuda_device):
    """Failure detection of the tensor-core kernels: with the pipeline wait limit lowered to 0
    (s4d_set_tc_wait_limit_ns) the barrier waits give up at once, the launch reports
    S4D_FLAG_WAIT_TIMEOUT in its error_flag and still finishes (each CTA waits for the copies and
    MMAs it issued before freeing tensor memory); with the limit restored, the next launches on
    the same context are correct and report nothing."""
    from sparse4d_tt_b200 import _lib as L

    dev = torch.device("cuda:0")
    gen = torch.Generator().manual_seed(11)
    rows, n, m, c = 28800, 416, 18, 256
    w_fc, w_kps, b_kps = _weights(n, m, c, gen, dev)
    inst = torch.randn(rows, c, generator=gen).to(dev)
    embed = torch.randn(rows, c, generator=gen).to(dev)
    w_o = ((torch.rand(c, c, generator=gen) * 2 - 1) * (3 / c) ** 0.5).to(dev)
    b_o = torch.randn(c, generator=gen).to(dev)
    logits = torch.empty(rows, n, device=dev)
    learn = torch.empty(rows, m, device=dev)
    out = torch.empty(rows, 2 * c, device=dev)
    lib = L.lib()
    flags = torch.zeros(2, dtype=torch.int32, device=dev)
    prev = lib.s4d_set_tc_wait_limit_ns(0)
    try:
        ops.weights_fc_into(logits, learn, inst, embed, w_fc, w_kps, b_kps, error_flag=flags[0:1])
        ops.output_proj_into(out, inst, w_o, b_o, embed, "cat", error_flag=flags[1:2])
    finally:
        lib.s4d_set_tc_wait_limit_ns(prev)
    torch.cuda.synchronize()
    assert prev == 2_000_000_000
    assert flags[0].item() & L.S4D_FLAG_WAIT_TIMEOUT and flags[1].item() & L.S4D_FLAG_WAIT_TIMEOUT
    flags.zero_()
    ops.weights_fc_into(logits, learn, inst, embed, w_fc, w_kps, b_kps, error_flag=flags[0:1])
    ops.output_proj_into(out, inst, w_o, b_o, embed, "cat", error_flag=flags[1:2])
    torch.cuda.synchronize()
    assert flags.tolist() == [0, 0]
    i64, e64, wf = inst.double(), embed.double(), w_fc.double()
    _check(logits, (i64 + e64) @ wf.T, (i64.abs() + e64.abs()) @ wf.abs().T, "logits after a timed-out launch")
    _check(out[:, :c], i64 @ w_o.double().T + b_o.double(), i64.abs() @ w_o.double().abs().T + 1e-6,
           "output_proj after a timed-out launch")
    assert torch.equal(out[:, c:], embed)


@pytest.mark.parametrize("mode", ["cat", "add", "none"])
@pytest.mark.parametrize("rows,row0,total", [(1, 0, 1), (129, 7, 300), (900, 900, 1800), (7200, 7200, 14400),
                                             (14400, 0, 28800)])
def test_output_proj_sum_of_two_sources(cuda_device, mode, rows, row0, total):
    """s4d_dfa_output_proj_sum: rows row0 .. row0 + rows - 1 of (features + features2), the sum
    formed by two MMAs per K step into one accumulator (here both sources are on this GPU; the
    camera-sharded mode passes a peer GPU's buffer as the second)."""
    dev = torch.device("cuda:0")
    gen = torch.Generator().manual_seed(rows + row0 + len(mode))
    c = 256
    w = ((torch.rand(c, c, generator=gen) * 2 - 1) * (3 / c) ** 0.5).to(dev)
    b = torch.randn(c, generator=gen).to(dev)
    f1 = torch.randn(total, c, generator=gen).to(dev)
    f2 = torch.randn(total, c, generator=gen).to(dev)
    inst_wide = torch.randn(rows, 2 * c, generator=gen).to(dev)
    inst = inst_wide[:, :c]
    width = 2 * c if mode == "cat" else c + 8
    out = torch.full((rows, width), -7.0, device=dev)
    flag = torch.zeros(1, dtype=torch.int32, device=dev)
    ops.output_proj_sum_into(out, f1, f2.data_ptr(), row0, rows, w, b, None if mode == "none" else inst, mode,
                             error_flag=flag)
    torch.cuda.synchronize()
    assert flag.item() == 0
    a64, b64, w64 = f1[row0:row0 + rows].double(), f2[row0:row0 + rows].double(), w.double()
    ref = (a64 + b64) @ w64.T + b.double()
    scale = (a64.abs() + b64.abs()) @ w64.abs().T + 1e-6
    if mode == "add":
        ref = ref + inst.double()
    _check(out[:, :c], ref, scale, f"output_proj_sum {mode} rows={rows} row0={row0}")
    if mode == "cat":
        assert torch.equal(out[:, c:], inst)
    else:
        assert torch.all(out[:, c:] == -7.0)


def test_output_proj_sum_with_zero_second_source_equals_output_proj(cuda_device):
    """With features2 all zeros the sum kernel gives output_proj's result bit for bit (adding
    exact zeros to the accumulator changes nothing)."""
    dev = torch.device("cuda:0")
    gen = torch.Generator().manual_seed(5)
    rows, c = 2700, 256
    w = ((torch.rand(c, c, generator=gen) * 2 - 1) * (3 / c) ** 0.5).to(dev)
    b = torch.randn(c, generator=gen).to(dev)
    f1 = torch.randn(2 * rows, c, generator=gen).to(dev)
    zeros = torch.zeros(2 * rows, c, device=dev)
    inst = torch.randn(rows, c, generator=gen).to(dev)
    got = torch.empty(rows, 2 * c, device=dev)
    ref = torch.empty(rows, 2 * c, device=dev)
    ops.output_proj_sum_into(got, f1, zeros.data_ptr(), rows, rows, w, b, inst, "cat")
    ops.output_proj_into(ref, f1[rows:].contiguous(), w, b, inst, "cat")
    torch.cuda.synchronize()
    assert torch.equal(got, ref)
