"""Parity of the sm_100a selective-scan kernels with the CPU oracle (float64).

Every case calls the kernels through the C ABI (swiftx_b200/_lib -> libswiftx_b200.so)
and compares with oracle.scan_fwd / oracle.scan_bwd on the same seeded inputs.

Tolerances: fp32 outputs rtol 1e-4 / atol 1e-5 (the reference's fast-vs-ref pin,
tests/test_selective_scan.py:74).  Gradients that are sums over many terms (dA, dD,
d delta_bias over b*L terms; dB, dC over D channels; dh0 over L steps) are compared with atol scaled
by the magnitude of what was summed (sum of |terms|, computed by the oracle on
|inputs|) times 1e-5, the fp32 re-association error of such sums.  bf16 inputs with
fp32 state: rtol 2e-2 against the oracle run on the same bf16-rounded values.
"""
import numpy as np
import pytest
import torch

import oracle
from swiftx_b200 import selective_scan_fast, selective_scan_fn, selective_scan_ref
from swiftx_b200.selective_scan import scan_backward, scan_forward
from swiftx_b200.triton_scan import selective_scan_triton
from swiftx_b200.workloads import config_inputs, reference_test_inputs

pytestmark = pytest.mark.gpu

DEV = "cuda"


def np64(t):
    return None if t is None else t.detach().cpu().double().numpy()


def assert_close(got, want, rtol, atol, name=""):
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    err = np.abs(got - want)
    bad = err > atol + rtol * np.abs(want)
    if bad.any():
        i = np.unravel_index(np.argmax(err - rtol * np.abs(want)), err.shape)
        raise AssertionError(f"{name}: {bad.sum()}/{bad.size} out of tolerance; worst at {i}: "
                             f"got {got[i]:.8g} want {want[i]:.8g} (max abs err {err.max():.3g})")


def oracle_case(inp, gate=True, softplus=True, with_D=True, h0=None):
    kw = dict(D=np64(inp["D"]) if with_D else None, z=np64(inp["z"]) if gate else None,
              delta_bias=np64(inp["delta_bias"]) if softplus else None, delta_softplus=softplus,
              h0=np64(h0))
    args = [np64(inp[k]) for k in ("u", "delta", "A", "B", "C")]
    out, hl = oracle.scan_fwd(*args, return_last_state=True, **kw)
    grads = oracle.scan_bwd(*args, np64(inp["dout"]), **kw)
    # magnitude scale of each reduction: the same sums over |terms|
    absargs = [np.abs(a) for a in args]
    absargs[2] = -absargs[2]                       # keep A negative (a decay)
    kwa = dict(kw)
    for k in ("D", "z"):
        if kwa[k] is not None:
            kwa[k] = np.abs(kwa[k])
    scale = oracle.scan_bwd(*absargs, np.abs(np64(inp["dout"])), **kwa)
    return out, hl, grads, scale


def check_grads(g, want, scale, rtol=1e-4, atol=1e-5):
    for k, v in want.items():
        if k in ("dA", "dD", "ddelta_bias", "dB", "dC", "dh0"):      # dh0: a sum over all L steps
            tol = atol + 1e-5 * np.abs(scale[k])
        else:
            tol = atol
        assert_close(np64(g[k]), v, rtol, tol, k)


# ----------------------------------------------------------------- golden fixtures
def test_golden_hand_tiny(golden):
    g = golden("hand_tiny")
    t = {k: torch.tensor(v, device=DEV, dtype=torch.float32) for k, v in g.items()}
    y = selective_scan_ref(t["u"], t["delta"], t["A"], t["B"], t["C"])
    assert_close(np64(y).ravel(), [2.0, 5.0, 8.5], 0, 1e-6, "y")


@pytest.mark.parametrize("L", [1, 7, 64])
def test_golden_forward(golden, L):
    g = golden(f"fwd_L{L}")
    t = {k: torch.tensor(v, device=DEV, dtype=torch.float32) for k, v in g.items()}
    for mode in ("auto", "parallel", "sequential", "fused", "triton"):
        y = selective_scan_fast(t["u"], t["delta"], t["A"], t["B"], t["C"], t["D"], mode=mode)
        assert_close(np64(y), g["y"], 1e-4, 1e-5, f"y[{mode}]")


@pytest.mark.parametrize("name", ["tail_2x37x40x16", "tail_1x20x8x5"])
def test_golden_tail_shapes_fwd_bwd(golden, name):
    g = golden(name)
    keys = ["u", "delta", "A", "B", "C"] + (["D"] if "D" in g else [])
    ins = [torch.tensor(g[k], device=DEV, dtype=torch.float32, requires_grad=True) for k in keys]
    y = selective_scan_triton(*ins, chunk=8)
    assert_close(np64(y), g["y"], 1e-4, 1e-4, "y")
    grads = torch.autograd.grad(y, ins, torch.tensor(g["gy"], device=DEV))
    for k, gr in zip(["du", "ddelta", "dA", "dB", "dC", "dD"], grads):
        # the reference's own Triton pin uses 2e-3 for grads (tests/test_triton_scan.py:30)
        assert_close(np64(gr), g[k], 1e-4, 1e-4, k)


def test_golden_gated_softplus(golden):
    g = golden("gated")
    keys = ["u", "delta_raw", "A", "B", "C", "D", "z", "delta_bias"]
    t = {k: torch.tensor(g[k], device=DEV, dtype=torch.float32, requires_grad=True) for k in keys}
    out = selective_scan_fn(t["u"], t["delta_raw"], t["A"], t["B"], t["C"], t["D"], z=t["z"],
                            delta_bias=t["delta_bias"], delta_softplus=True)
    assert_close(np64(out), g["out"], 1e-4, 1e-5, "out")
    grads = torch.autograd.grad(out, [t[k] for k in keys], torch.tensor(g["gout"], device=DEV))
    names = ["du", "ddelta", "dA", "dB", "dC", "dD", "dz", "ddelta_bias"]
    for k, gr in zip(names, grads):
        assert_close(np64(gr), g[k], 1e-4, 1e-4, k)


def test_golden_cpu_sized_forward(golden):
    g = golden("fwd_b2_L256_D128")
    t = {k: torch.tensor(v, device=DEV, dtype=torch.float32) for k, v in g.items()}
    y = selective_scan_fn(t["u"], t["delta_raw"], t["A"], t["B"], t["C"], t["D"],
                          delta_bias=t["delta_bias"], delta_softplus=True)
    assert_close(np64(y), g["y"], 1e-4, 1e-5, "y")


# ----------------------------------------------------------------- oracle parity
CASES = [
    # b, L, D, N, gate, softplus, with_D
    (2, 256, 128, 16, True, True, True),
    (1, 100, 40, 16, True, True, True),       # L not a multiple of 16/64, D not of 32
    (3, 33, 64, 5, False, False, True),       # N < 16, no gate, plain delta
    (2, 17, 24, 16, True, False, False),      # no D skip
    (1, 1, 32, 16, True, True, True),         # single step
    (2, 300, 96, 8, False, True, True),
]


@pytest.mark.parametrize("case", CASES)
def test_fwd_bwd_vs_oracle(case):
    b, L, D, N, gate, sp, wD = case
    inp = config_inputs(b, L, D, N, seed=b * 1000 + L, gate=gate, device=DEV)
    if not sp:   # plain delta: pass the positive softplus(delta_raw + bias) as the block does
        inp["delta"] = torch.nn.functional.softplus(inp["delta"] + inp["delta_bias"])
    out_o, hl_o, gr_o, scale = oracle_case(inp, gate, sp, wD)
    pre = torch.empty(inp["u"].shape, device=DEV, dtype=torch.float32)
    out, ck, hl = scan_forward(inp["u"], inp["delta"], inp["A"], inp["B"], inp["C"],
                               inp["D"] if wD else None, inp["z"] if gate else None,
                               inp["delta_bias"] if sp else None, sp, checkpoints=True,
                               return_last_state=True, pre_out=pre)
    assert_close(np64(out), out_o, 1e-4, 1e-5, "out")
    assert_close(np64(hl), hl_o, 1e-4, 1e-5, "h_last")
    args = (inp["u"], inp["delta"], inp["A"], inp["B"], inp["C"], inp["D"] if wD else None,
            inp["z"] if gate else None, inp["delta_bias"] if sp else None, sp, None, ck, inp["dout"])
    # backward with the saved pre-gate output and with the readout recomputed
    for y_pre in ((pre, None) if gate else (None,)):
        g = scan_backward(*args, y_pre=y_pre)
        check_grads({k: v for k, v in g.items() if v is not None}, gr_o, scale)


def test_initial_state_and_grad():
    b, L, D, N = 2, 50, 32, 16
    inp = config_inputs(b, L, D, N, seed=11, device=DEV)
    h0 = torch.randn(b, D, N, generator=torch.Generator().manual_seed(12)).to(DEV) * 0.3
    out_o, hl_o, gr_o, scale = oracle_case(inp, True, True, True, h0=h0)
    args = {k: inp[k].clone().requires_grad_() for k in ("u", "delta", "A", "B", "C", "D", "z", "delta_bias")}
    h0r = h0.clone().requires_grad_()
    out, hl = selective_scan_fn(args["u"], args["delta"], args["A"], args["B"], args["C"], args["D"],
                                z=args["z"], delta_bias=args["delta_bias"], delta_softplus=True,
                                h0=h0r, return_last_state=True)
    assert_close(np64(out), out_o, 1e-4, 1e-5, "out")
    assert_close(np64(hl), hl_o, 1e-4, 1e-5, "h_last")
    out.backward(inp["dout"])
    assert h0r.grad is not None and torch.isfinite(h0r.grad).all()
    oh = oracle.scan_bwd(*[np64(inp[k]) for k in ("u", "delta", "A", "B", "C")], np64(inp["dout"]),
                         D=np64(inp["D"]), z=np64(inp["z"]), delta_bias=np64(inp["delta_bias"]),
                         delta_softplus=True, h0=np64(h0))
    assert_close(np64(h0r.grad), oh["dh0"], 1e-4, 1e-5, "dh0")


def test_strided_inputs_match_contiguous():
    """x and z as the two halves of one (b, L, 2D) in_proj output (models/sift_block.py:115)."""
    b, L, D, N = 2, 70, 64, 16
    inp = config_inputs(b, L, D, N, seed=3, device=DEV)
    xz = torch.cat([inp["u"], inp["z"]], dim=-1)
    u_v, z_v = xz.chunk(2, dim=-1)
    assert u_v.stride(1) == 2 * D
    a = selective_scan_fn(u_v, inp["delta"], inp["A"], inp["B"], inp["C"], inp["D"], z=z_v,
                          delta_bias=inp["delta_bias"], delta_softplus=True)
    c = selective_scan_fn(inp["u"], inp["delta"], inp["A"], inp["B"], inp["C"], inp["D"], z=inp["z"],
                          delta_bias=inp["delta_bias"], delta_softplus=True)
    assert torch.equal(a, c)


def test_deterministic_backward():
    b, L, D, N = 2, 128, 96, 16
    inp = config_inputs(b, L, D, N, seed=4, device=DEV)
    args = (inp["u"], inp["delta"], inp["A"], inp["B"], inp["C"], inp["D"], inp["z"], inp["delta_bias"], True)
    _, ck, _ = scan_forward(*args, checkpoints=True)
    g1 = scan_backward(*args, None, ck, inp["dout"])
    g2 = scan_backward(*args, None, ck, inp["dout"])
    for k in g1:
        if g1[k] is not None:
            assert torch.equal(g1[k], g2[k]), k


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16], ids=["fp32", "bf16"])
def test_a_log_formed_in_kernel_matches_torch_chain(dtype):
    """A_is_log=True (the kernels form A = -exp(A_log) and return d/dA_log) against the
    block's torch expression A = -torch.exp(A_log) feeding the plain call, through
    autograd: the same values (the kernel's expf is the function torch.exp evaluates), so
    outputs and every gradient agree to rounding; a 1x2 channel tail and N < 16 included."""
    b, L, D, N = 2, 77, 66, 12
    inp = config_inputs(b, L, D, N, seed=11, device=DEV, dtype=dtype)
    g = torch.Generator(device="cpu").manual_seed(3)
    A_log = (torch.log(torch.arange(1, N + 1, dtype=torch.float32)).repeat(D, 1)
             + 0.1 * torch.randn(D, N, generator=g)).to(DEV)
    keys = ["u", "delta", "B", "C", "D", "z", "delta_bias"]
    res = []
    for in_kernel in (False, True):
        t = {k: inp[k].clone().requires_grad_() for k in keys}
        al = A_log.clone().requires_grad_()
        A = al if in_kernel else -torch.exp(al)
        out = selective_scan_fn(t["u"], t["delta"], A, t["B"], t["C"], t["D"], z=t["z"],
                                delta_bias=t["delta_bias"], delta_softplus=True, A_is_log=in_kernel)
        out.backward(inp["dout"])
        res.append((out.detach(), al.grad, {k: t[k].grad for k in keys}))
    (o0, a0, g0), (o1, a1, g1) = res
    assert_close(np64(o1), np64(o0), 1e-6, 1e-7, "out")
    assert_close(np64(a1), np64(a0), 1e-6, 1e-6 * float(a0.abs().max()), "dA_log")
    for k in keys:
        assert_close(np64(g1[k]), np64(g0[k]), 1e-6, 1e-6 * float(g0[k].abs().max()), k)


def test_bf16_inputs_fp32_state():
    b, L, D, N = 2, 200, 64, 16
    inp = config_inputs(b, L, D, N, seed=9, device=DEV, dtype=torch.bfloat16)
    out, _, _ = scan_forward(inp["u"], inp["delta"], inp["A"], inp["B"], inp["C"], inp["D"], inp["z"],
                             inp["delta_bias"], True, out_dtype=torch.float32)
    assert out.dtype == torch.float32
    want = oracle.scan_fwd(*[np64(inp[k]) for k in ("u", "delta", "A", "B", "C")], D=np64(inp["D"]),
                           z=np64(inp["z"]), delta_bias=np64(inp["delta_bias"]), delta_softplus=True)
    assert_close(np64(out), want, 2e-2, 1e-3, "out")


def test_cpu_tensors_raise():
    u, delta, A, B, C, Ds = reference_test_inputs(2, 6, 3, 4)
    with pytest.raises(RuntimeError):
        selective_scan_fast(u, delta, A, B, C, Ds)


def test_full_size_8x2048x512_vs_oracle():
    """The benchmark configuration itself (b=8, L=2048, D=512, N=16, gated, softplus)."""
    inp = config_inputs(8, 2048, 512, 16, seed=0, device=DEV)
    oracle.set_num_threads(max(1, oracle.num_threads()))
    out_o, hl_o, gr_o, scale = oracle_case(inp)
    pre = torch.empty(inp["u"].shape, device=DEV, dtype=torch.float32)
    out, ck, _ = scan_forward(inp["u"], inp["delta"], inp["A"], inp["B"], inp["C"], inp["D"], inp["z"],
                              inp["delta_bias"], True, checkpoints=True, pre_out=pre)
    assert_close(np64(out), out_o, 1e-4, 1e-5, "out")
    g = scan_backward(inp["u"], inp["delta"], inp["A"], inp["B"], inp["C"], inp["D"], inp["z"],
                      inp["delta_bias"], True, None, ck, inp["dout"], y_pre=pre)
    check_grads({k: v for k, v in g.items() if v is not None}, gr_o, scale)


def _bwd_path(inp, use_pre):
    """(segments, CTAs per SM) of swx_scan_bwd for these inputs: segments 0 = row kernel."""
    from swiftx_b200 import _lib
    from swiftx_b200.selective_scan import _fill_inputs, _prep
    args = (inp["u"], inp["delta"], inp["A"], inp["B"], inp["C"], inp["D"], inp["z"], inp["delta_bias"], True)
    a = _lib.ScanArgs()
    u, dl, A, Bm, Cm, Dv, z, bias, h0, in_dt = _prep(*args[:8], None)
    _fill_inputs(a, u, dl, A, Bm, Cm, Dv, z, bias, h0, True, in_dt)
    a.out_pre = 16 if (use_pre and z is not None) else None          # only its presence matters here
    lib = _lib.load()
    return lib.swx_scan_bwd_segments(a), lib.swx_scan_bwd_ctas_per_sm(a)


def _run_bwd(inp, use_pre):
    args = (inp["u"], inp["delta"], inp["A"], inp["B"], inp["C"], inp["D"], inp["z"], inp["delta_bias"], True)
    pre = torch.empty(inp["u"].shape, device=DEV, dtype=torch.float32) if use_pre else None
    _, ck, _ = scan_forward(*args, checkpoints=True, pre_out=pre)
    return scan_backward(*args, None, ck, inp["dout"], y_pre=pre)


@pytest.mark.parametrize("shape,gate,use_pre", [((5, 100, 1024, 16), True, True),
                                                ((5, 100, 1024, 16), True, False),
                                                ((10, 37, 520, 5), False, False),
                                                ((16, 1024, 128, 16), True, True)])
def test_bwd_batch_split_bit_identical(shape, gate, use_pre):
    """fp32 inputs (the time-segmented backward), with and without the saved pre-gate
    output, N < 16 and a partial last channel block: its segment plan depends on (L, D)
    and counts at most 8 rows (short sequences get one segment whatever the batch), so
    each row's per-row gradients are bit-identical whether the rows are passed together
    or in two smaller batches -- at 16 rows split 8 + 8, 8 segments each; the batch sums
    agree to fp32 re-association, and everything matches the oracle."""
    b, L, D, N = shape
    inp = config_inputs(b, L, D, N, seed=41, gate=gate, device=DEV)
    rowwise = ("u", "delta", "z", "B", "C", "dout")
    cut = {5: 2, 10: 4, 16: 8}[b]
    sub = lambda rows: {k: (v[rows] if k in rowwise and v is not None else v) for k, v in inp.items()}  # noqa: E731
    paths = {_bwd_path(sub(r), use_pre) for r in (slice(0, b), slice(0, cut), slice(cut, b))}
    assert len(paths) == 1 and next(iter(paths))[0] >= 1          # one segmented plan for all three
    g_all, g_a, g_b = _run_bwd(sub(slice(0, b)), use_pre), _run_bwd(sub(slice(0, cut)), use_pre), \
        _run_bwd(sub(slice(cut, b)), use_pre)
    for k in ("du", "ddelta", "dz", "dB", "dC"):
        if g_all[k] is not None:
            assert torch.equal(g_all[k], torch.cat([g_a[k], g_b[k]])), k
    for k in ("dA", "dD", "ddelta_bias"):
        want = (g_a[k] + g_b[k]).double().cpu().numpy()
        np.testing.assert_allclose(np64(g_all[k]), want, rtol=1e-5, atol=1e-5 * np.abs(want).max(), err_msg=k)
    _, _, gr_o, scale = oracle_case(inp, gate=gate)
    check_grads({k: v for k, v in g_all.items() if v is not None}, gr_o, scale)


@pytest.mark.parametrize("shape,gate,use_pre", [((5, 100, 1024, 16), True, True),
                                                ((5, 100, 1024, 16), True, False),
                                                ((10, 37, 520, 5), False, False),
                                                ((16, 64, 512, 16), True, True)])
def test_bwd_row_kernel_bf16_vs_oracle(shape, gate, use_pre):
    """bf16 problems whose 32-channel x row grid fills every SM (two CTAs each) run the
    whole-row backward kernel (the Sift LM block's shape among them): against the oracle at
    the bf16 tolerance, rtol 2e-2 with atol 2e-2 of each gradient's magnitude."""
    inp = config_inputs(*shape, seed=41, gate=gate, device=DEV, dtype=torch.bfloat16)
    assert _bwd_path(inp, use_pre) == (0, 2)
    g = _run_bwd(inp, use_pre)
    _, _, gr_o, scale = oracle_case(inp, gate=gate)
    for k in ("du", "ddelta", "dz", "dB", "dC", "dA", "dD", "ddelta_bias"):
        if k not in gr_o:
            continue
        want = gr_o[k]
        assert_close(np64(g[k]), want, 2e-2, 2e-2 * np.abs(want).max() + 1e-5 * np.abs(scale[k]).max(), k)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16], ids=["fp32", "bf16"])
def test_bwd_many_segments_vs_oracle(dtype):
    """A long sequence over few channels: the backward walks it as several time segments
    (carries from 16-step sub-segment summaries), with a tail chunk, an initial state and
    its gradient; against the oracle (fp32 1e-4 / bf16 2e-2)."""
    b, L, D, N = 2, 1000, 64, 16
    inp = config_inputs(b, L, D, N, seed=17, device=DEV, dtype=dtype)
    assert _bwd_path(inp, True)[0] >= 4
    h0 = (torch.randn(b, D, N, generator=torch.Generator().manual_seed(5)) * 0.3).to(DEV)
    out_o, hl_o, gr_o, scale = oracle_case(inp, h0=h0)
    pre = torch.empty(inp["u"].shape, device=DEV, dtype=torch.float32)
    out, ck, _ = scan_forward(inp["u"], inp["delta"], inp["A"], inp["B"], inp["C"], inp["D"], inp["z"],
                              inp["delta_bias"], True, h0=h0, checkpoints=True, pre_out=pre)
    g = scan_backward(inp["u"], inp["delta"], inp["A"], inp["B"], inp["C"], inp["D"], inp["z"],
                      inp["delta_bias"], True, h0, ck, inp["dout"], y_pre=pre)
    g = {k: v for k, v in g.items() if v is not None}
    if dtype == torch.float32:
        check_grads(g, gr_o, scale)
    else:
        for k, want in gr_o.items():
            assert_close(np64(g[k]), want, 2e-2, 2e-2 * np.abs(want).max() + 1e-5 * np.abs(scale.get(k, 0)).max(), k)


# ----------------------------------------------------------------- float64 inputs
def _ref_inputs_f64(b=2, L=6, D=3, N=4, seed=0):
    """The reference suite's generator (tests/test_selective_scan.py:14-22) in float64 on
    the GPU."""
    return [t.double().to(DEV) for t in reference_test_inputs(b, L, D, N, seed=seed)]


def test_float64_returns_float64_and_matches_golden(golden):
    """float64 in -> float64 out and float64 gradients, computed in float64: the golden
    float64 backward made by the reference (tests/test_selective_scan.py:77-86 shapes)
    at the reference's own pin (atol 1e-9, rtol 1e-7)."""
    g = golden("bwd_f64")
    keys = ["u", "delta", "A", "B", "C", "D"]
    t = [torch.tensor(g[k], device=DEV, dtype=torch.float64, requires_grad=True) for k in keys]
    y = selective_scan_fast(*t)
    assert y.dtype == torch.float64
    np.testing.assert_allclose(np64(y), g["y"], rtol=1e-7, atol=1e-9)
    (y * torch.tensor(g["gy"], device=DEV)).sum().backward()
    for k, ti in zip(["du", "ddelta", "dA", "dB", "dC", "dD"], t):
        assert ti.grad.dtype == torch.float64, k
        np.testing.assert_allclose(ti.grad.detach().cpu().numpy(), g[k], rtol=1e-7, atol=1e-9, err_msg=k)


@pytest.mark.parametrize("mode", ["auto", "parallel", "sequential", "fused", "triton"])
def test_float64_gradcheck(mode):
    """torch.autograd.gradcheck through the drop-in on CUDA float64 tensors, as the
    reference checks its own modes (tests/test_selective_scan.py:89-93)."""
    tensors = [t.requires_grad_() for t in _ref_inputs_f64()]
    fn = lambda *t: selective_scan_fast(*t, mode=mode)  # noqa: E731
    assert torch.autograd.gradcheck(fn, tensors)


def test_float64_gradcheck_gated_softplus_initial_state():
    """The extended entry point in float64: gate, softplus(delta + bias), D skip, an
    initial state and A given as its log, all gradients checked by finite differences."""
    g = torch.Generator().manual_seed(5)
    b, L, D, N = 2, 19, 3, 4
    mk = lambda *s, sc=1.0: (torch.randn(*s, generator=g) * sc).double().to(DEV).requires_grad_()  # noqa: E731
    u, dr, z = mk(b, L, D), mk(b, L, D, sc=0.5), mk(b, L, D)
    Bm, Cm = mk(b, L, N), mk(b, L, N)
    A_log = (torch.rand(D, N, generator=g) * 0.5).double().to(DEV).requires_grad_()
    Dsk, bias, h0 = mk(D), mk(D, sc=0.3), mk(b, D, N, sc=0.3)
    fn = lambda *a: selective_scan_fn(a[0], a[1], a[2], a[3], a[4], a[5], z=a[6], delta_bias=a[7],  # noqa: E731
                                      delta_softplus=True, h0=a[8], A_is_log=True)
    assert torch.autograd.gradcheck(fn, (u, dr, A_log, Bm, Cm, Dsk, z, bias, h0))


def test_float64_long_sequence_vs_oracle():
    """float64 over several 16-step checkpoint chunks and more than one channel block,
    against the oracle at the float64 pin."""
    inp = config_inputs(2, 150, 70, 16, seed=8, device=DEV, dtype=torch.float64)
    for k in ("A", "D", "delta_bias"):
        inp[k] = inp[k].double()
    out_o, hl_o, gr_o, _ = oracle_case(inp)
    out, ck, hl = scan_forward(inp["u"], inp["delta"], inp["A"], inp["B"], inp["C"], inp["D"], inp["z"],
                               inp["delta_bias"], True, checkpoints=True, return_last_state=True)
    assert out.dtype == torch.float64 and hl.dtype == torch.float64
    np.testing.assert_allclose(np64(out), out_o, rtol=1e-9, atol=1e-11)
    g = scan_backward(inp["u"], inp["delta"], inp["A"], inp["B"], inp["C"], inp["D"], inp["z"],
                      inp["delta_bias"], True, None, ck, inp["dout"])
    for k, v in gr_o.items():
        np.testing.assert_allclose(g[k].detach().cpu().numpy(), v, rtol=1e-9, atol=1e-9 * np.abs(v).max(),
                                   err_msg=k)


@pytest.mark.parametrize("shape", [(2, 0, 64), (0, 50, 64)], ids=["L=0", "b=0"])
def test_empty_problems(shape):
    """An empty sequence or batch: empty outputs, the final state equal to h0 (nothing
    decays it), and zero gradients for the parameters and h0 (nothing depends on them),
    as the reference's expressions give."""
    b, L, D = shape
    N = 16
    g = torch.Generator(device=DEV).manual_seed(3)
    t = lambda *s: torch.randn(*s, device=DEV, generator=g).requires_grad_()  # noqa: E731
    u, dl, z = t(b, L, D), t(b, L, D), t(b, L, D)
    Bm, Cm = t(b, L, N), t(b, L, N)
    A = (-torch.rand(D, N, device=DEV, generator=g) - 0.1).requires_grad_()
    Dv, bias, h0 = t(D), t(D), t(b, D, N)
    out, hl = selective_scan_fn(u, dl, A, Bm, Cm, Dv, z=z, delta_bias=bias, delta_softplus=True, h0=h0,
                                return_last_state=True)
    assert out.shape == (b, L, D)
    if L == 0:
        assert torch.equal(hl, h0.detach())
    out.sum().backward()
    for name, p in (("A", A), ("D", Dv), ("delta_bias", bias), ("h0", h0)):
        assert p.grad is not None and torch.equal(p.grad, torch.zeros_like(p)), name
