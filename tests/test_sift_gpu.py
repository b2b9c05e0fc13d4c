"""The Sift block / LM running on the B200 kernels, tested the way the reference tests
its block and model (tests/test_sift_block.py, tests/test_model.py): shapes, causality,
recurrent step == parallel forward, gradients reach every parameter, a tiny batch
overfits.  Block parity: the whole block is recomputed on the CPU with the oracle for
the scan and conv and torch for the projections."""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

import oracle
from swiftx_b200.sift import SiftBlock, SiftConfig, SiftLM, count_params

pytestmark = pytest.mark.gpu
DEV = "cuda"


def make_block(**kw):
    torch.manual_seed(0)
    return SiftBlock(d_model=16, d_state=8, d_conv=4, expand=2, **kw).to(DEV)


def block_oracle(blk, hidden):
    """The reference block's forward (models/sift_block.py:111-135), with the oracle
    for conv + scan, on float64 CPU copies of the parameters."""
    p = {k: v.detach().double().cpu() for k, v in blk.state_dict().items()}
    h = hidden.detach().double().cpu()
    xz = h @ p["in_proj.weight"].T
    D = blk.d_inner
    x, z = xz[..., :D], xz[..., D:]
    xc = torch.from_numpy(oracle.conv1d_fwd(x.numpy(), p["conv1d.weight"].numpy(), p["conv1d.bias"].numpy()))
    x_dbl = xc @ p["x_proj.weight"].T
    dt, B, C = torch.split(x_dbl, [blk.dt_rank, blk.d_state, blk.d_state], dim=-1)
    delta = F.softplus(dt @ p["dt_proj.weight"].T + p["dt_proj.bias"])
    A = -torch.exp(p["A_log"])
    y = oracle.scan_fwd(xc.numpy(), delta.numpy(), A.numpy(), B.numpy(), C.numpy(), p["D"].numpy(),
                        z=z.numpy())
    return torch.from_numpy(y) @ p["out_proj.weight"].T


def test_shapes_and_dims():
    blk = make_block()
    assert blk.d_inner == 32 and blk.dt_rank == 1
    assert blk(torch.randn(2, 10, 16, device=DEV)).shape == (2, 10, 16)


def test_block_matches_oracle():
    blk = make_block()
    x = torch.randn(2, 37, 16, device=DEV)
    np.testing.assert_allclose(blk(x).detach().double().cpu().numpy(), block_oracle(blk, x).numpy(),
                               rtol=1e-4, atol=1e-5)


def test_state_dict_keys_match_reference_layout():
    keys = set(make_block().state_dict())
    assert keys == {"in_proj.weight", "conv1d.weight", "conv1d.bias", "x_proj.weight", "dt_proj.weight",
                    "dt_proj.bias", "A_log", "D", "out_proj.weight"}
    assert make_block().conv1d.weight.shape == (32, 1, 4)


def test_causal_no_future_leak():
    blk = make_block()
    x = torch.randn(1, 20, 16, device=DEV)
    y1 = blk(x)
    x2 = x.clone()
    x2[:, 13:] = torch.randn(1, 7, 16, device=DEV)
    y2 = blk(x2)
    assert torch.allclose(y1[:, :13], y2[:, :13], atol=1e-6)
    assert not torch.allclose(y1[:, 13:], y2[:, 13:])


def test_step_matches_forward():
    blk = make_block()
    x = torch.randn(2, 9, 16, device=DEV)
    y_full = blk(x)
    state = blk.allocate_state(2, device=DEV)
    ys = [blk.step(x[:, t], state) for t in range(9)]
    assert torch.allclose(y_full, torch.stack(ys, 1), atol=1e-5)


def test_gradients_reach_all_parameters():
    blk = make_block()
    blk(torch.randn(2, 8, 16, device=DEV)).pow(2).sum().backward()
    for name, p in blk.named_parameters():
        assert p.grad is not None and torch.isfinite(p.grad).all(), name
        assert p.grad.abs().sum() > 0, name


def test_block_grads_match_autograd_oracle():
    """Gradients of the kernel block vs torch autograd through a float64 reference block
    built from the oracle's fused-scan definition (conv via F.conv1d, scan via a loop)."""
    blk = make_block()
    x = torch.randn(2, 12, 16, device=DEV)
    blk(x).pow(2).sum().backward()
    p = {k: v.detach().double().cpu().requires_grad_() for k, v in blk.state_dict().items()}
    h = x.double().cpu()
    xz = h @ p["in_proj.weight"].T
    D = blk.d_inner
    xx, z = xz[..., :D], xz[..., D:]
    L = xx.shape[1]
    xc = F.silu(F.conv1d(xx.transpose(1, 2), p["conv1d.weight"], p["conv1d.bias"], padding=3,
                         groups=D)[..., :L].transpose(1, 2))
    dt, B, C = torch.split(xc @ p["x_proj.weight"].T, [blk.dt_rank, blk.d_state, blk.d_state], dim=-1)
    delta = F.softplus(dt @ p["dt_proj.weight"].T + p["dt_proj.bias"])
    A = -torch.exp(p["A_log"])
    hst = torch.zeros(2, D, blk.d_state, dtype=torch.float64)
    ys = []
    for t in range(L):
        hst = torch.exp(delta[:, t, :, None] * A) * hst + delta[:, t, :, None] * B[:, t, None, :] * xc[:, t, :, None]
        ys.append((hst * C[:, t, None, :]).sum(-1))
    y = (torch.stack(ys, 1) + xc * p["D"]) * F.silu(z)
    (y @ p["out_proj.weight"].T).pow(2).sum().backward()
    got = dict(blk.named_parameters())
    for k, v in p.items():
        np.testing.assert_allclose(got[k].grad.double().cpu().numpy(), v.grad.numpy(), rtol=1e-3, atol=1e-4,
                                   err_msg=k)


def tiny_cfg(**kw):
    return SiftConfig(vocab_size=11, d_model=32, n_layers=2, d_state=8, **kw)


def test_lm_forward_shapes_and_loss():
    torch.manual_seed(0)
    m = SiftLM(tiny_cfg()).to(DEV)
    idx = torch.randint(0, 11, (3, 15), device=DEV)
    logits, loss = m(idx, torch.randint(0, 11, (3, 15), device=DEV))
    assert logits.shape == (3, 15, 11)
    assert abs(loss.item() - np.log(11.0)) < 0.3
    assert m.lm_head.weight.data_ptr() == m.embedding.weight.data_ptr() and count_params(m) > 0


def test_lm_recurrent_step_matches_parallel_forward():
    torch.manual_seed(0)
    m = SiftLM(tiny_cfg()).to(DEV).eval()
    idx = torch.randint(0, 11, (2, 12), device=DEV)
    logits, _ = m(idx)
    state = m.allocate_state(2, device=DEV)
    steps = torch.stack([m.step(idx[:, t], state) for t in range(12)], 1)
    assert torch.allclose(logits, steps, atol=1e-4)


def test_lm_overfits_tiny_batch():
    torch.manual_seed(0)
    m = SiftLM(tiny_cfg()).to(DEV)
    idx = torch.randint(0, 11, (4, 16), device=DEV)
    opt = torch.optim.AdamW(m.parameters(), lr=3e-3)
    first = None
    for _ in range(150):
        _, loss = m(idx[:, :-1], idx[:, 1:])
        first = first or loss.item()
        opt.zero_grad()
        loss.backward()
        opt.step()
    assert loss.item() < 0.1 * first


def test_generate_length():
    m = SiftLM(tiny_cfg()).to(DEV)
    out = m.generate(torch.zeros(2, 3, dtype=torch.long, device=DEV), 5, temperature=0)
    assert out.shape == (2, 8)


@pytest.mark.parametrize("accumulate", [True, False], ids=["accumulate", "assign"])
def test_graph_captured_train_step_matches_eager(accumulate):
    """The training step replayed from CUDA graphs (forward+backward, then clip+AdamW)
    follows the same loss trajectory as the eager step (the kernels launch on the
    capturing stream and allocate from the graph's pool), with the gradients accumulated
    into a flat buffer's views and with them assigned by the backward (bench.py's LM
    step), where the update graph reads the gradients from the first graph's pool."""
    from swiftx_b200.data_parallel import FlatGradients

    def run(graphed):
        torch.manual_seed(0)
        m = SiftLM(tiny_cfg()).to(DEV)
        params = list(m.parameters())
        grads = FlatGradients(params, accumulate=accumulate)
        opt = torch.optim.AdamW(params, lr=3e-3, fused=True, capturable=graphed)
        idx = torch.randint(0, 11, (4, 17), device=DEV, generator=torch.Generator(device=DEV).manual_seed(1))

        def fwd_bwd():
            grads.zero_()
            _, loss = m(idx[:, :-1], idx[:, 1:])
            loss.backward()
            grads.pack_()
            return loss.detach()

        def update():
            torch.nn.utils.clip_grad_norm_(params, 1.0)
            opt.step()

        losses = []
        if graphed:
            side = torch.cuda.Stream()
            side.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(side):
                losses.append(fwd_bwd().item())
                update()
            torch.cuda.current_stream().wait_stream(side)
            g1, g2 = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
            with torch.cuda.graph(g1):
                static_loss = fwd_bwd()
            with torch.cuda.graph(g2):
                update()
            for _ in range(40):
                g1.replay()
                losses.append(static_loss.item())
                g2.replay()
        else:
            for _ in range(41):
                losses.append(fwd_bwd().item())
                update()
        return losses

    eager, graphed = run(False), run(True)
    assert graphed[-1] < 0.5 * graphed[0]
    np.testing.assert_allclose(graphed[:10], eager[:10], rtol=1e-3)


def test_bf16_weight_copies_match_autocast():
    """SiftLM under bf16 autocast with its per-forward bf16 weight copies (_Bf16Linear)
    against plain autocast: the same bf16 GEMMs, so identical logits; gradients agree to
    bf16 rounding (autocast rounds each projection's weight gradient to bf16 before casting
    it back to fp32, the copies' path returns the GEMM's fp32 result)."""
    torch.manual_seed(0)
    m = SiftLM(SiftConfig(vocab_size=64, d_model=128, n_layers=2, d_state=16)).to(DEV)
    tok = torch.randint(0, 64, (2, 97), device=DEV)

    def run(copies):
        m.bf16_weight_copies = copies
        m.zero_grad(set_to_none=True)
        with torch.autocast("cuda", dtype=torch.bfloat16):
            logits, loss = m(tok[:, :-1], tok[:, 1:])
        loss.backward()
        return logits.detach().float(), {n: p.grad.clone() for n, p in m.named_parameters()}

    l1, g1 = run(True)
    l0, g0 = run(False)
    assert torch.equal(l1, l0)
    for n in g0:
        assert g1[n].dtype == torch.float32, n
        tol = 2e-2 * float(g0[n].abs().max())
        np.testing.assert_allclose(g1[n].cpu().numpy(), g0[n].cpu().numpy(), rtol=2e-2, atol=tol, err_msg=n)


def test_fused_mixer_core_matches_per_op_graph():
    """The mixer between in_proj and out_proj as one autograd node (_MixerCore: dz and the
    conv's dx written into the two halves of one d(xz) buffer, the scan's du added inside
    x_proj's input-gradient GEMM) against the per-op graph of the same kernels: identical
    logits (the forward runs the same kernels and GEMMs), gradients equal to bf16 rounding
    (the fused add rounds once instead of twice)."""
    from swiftx_b200 import sift as sift_mod
    torch.manual_seed(0)
    m = SiftLM(SiftConfig(vocab_size=64, d_model=128, n_layers=2, d_state=16)).to(DEV)
    tok = torch.randint(0, 64, (3, 130), device=DEV)

    def run(fused):
        prev = sift_mod._FUSED_CORE
        sift_mod._FUSED_CORE = fused
        try:
            m.zero_grad(set_to_none=True)
            with torch.autocast("cuda", dtype=torch.bfloat16):
                logits, loss = m(tok[:, :-1], tok[:, 1:])
            loss.backward()
        finally:
            sift_mod._FUSED_CORE = prev
        return logits.detach().float(), {n: p.grad.clone() for n, p in m.named_parameters()}

    l1, g1 = run(True)
    l0, g0 = run(False)
    assert torch.equal(l1, l0)
    assert set(g1) == set(g0)
    for n in g0:
        assert g1[n].dtype == g0[n].dtype and g1[n].shape == g0[n].shape, n
        tol = 2e-2 * float(g0[n].abs().max())
        np.testing.assert_allclose(g1[n].cpu().numpy(), g0[n].cpu().numpy(), rtol=2e-2, atol=tol, err_msg=n)


def make_pathway_block():
    """SiftX block: three timescale groups over 32 channels (sizes 11/10/11) and the
    per-token pathway gate, with non-zero pathway weights so the mix is not the identity."""
    torch.manual_seed(0)
    blk = SiftBlock(d_model=16, d_state=8, d_conv=4, expand=2, timescales=[(1e-3, 1e-2), (1e-2, 3e-2), (3e-2, 1e-1)],
                    pathway_gate=True).to(DEV)
    with torch.no_grad():
        blk.pathway.weight.normal_(0, 0.5)
        blk.pathway.bias.normal_(0, 0.5)
    return blk


def _pathway_reference(blk, hidden, scan):
    """models/sift_block.py:111-142 with pathway mixing, float64 on the CPU; `scan` computes
    the ungated scan y + D*u from (xc, delta, A, B, C, D)."""
    p = {k: v.detach().double().cpu() for k, v in blk.state_dict().items()}
    h = hidden.detach().double().cpu()
    xz = h @ p["in_proj.weight"].T
    D = blk.d_inner
    x, z = xz[..., :D], xz[..., D:]
    L = x.shape[1]
    xc = F.silu(F.conv1d(x.transpose(1, 2), p["conv1d.weight"], p["conv1d.bias"], padding=3,
                         groups=D)[..., :L].transpose(1, 2))
    dt, B, C = torch.split(xc @ p["x_proj.weight"].T, [blk.dt_rank, blk.d_state, blk.d_state], dim=-1)
    delta = F.softplus(dt @ p["dt_proj.weight"].T + p["dt_proj.bias"])
    A = -torch.exp(p["A_log"])
    y = scan(xc, delta, A, B, C, p["D"])
    w = torch.softmax(xc @ p["pathway.weight"].T + p["pathway.bias"], dim=-1) * blk.n_groups
    y = y * w[..., blk.group_of.cpu()] * F.silu(z)
    return y @ p["out_proj.weight"].T


def test_pathway_block_matches_oracle():
    blk = make_pathway_block()
    assert blk.group_of.tolist() == [0] * 11 + [1] * 10 + [2] * 11
    x = torch.randn(2, 29, 16, device=DEV)

    def scan(xc, delta, A, B, C, Dv):
        return torch.from_numpy(oracle.scan_fwd(xc.numpy(), delta.numpy(), A.numpy(), B.numpy(), C.numpy(),
                                                Dv.numpy()))
    np.testing.assert_allclose(blk(x).detach().double().cpu().numpy(), _pathway_reference(blk, x, scan).numpy(),
                               rtol=1e-4, atol=1e-5)


def test_pathway_step_matches_forward():
    blk = make_pathway_block()
    x = torch.randn(2, 9, 16, device=DEV)
    y_full = blk(x)
    state = blk.allocate_state(2, device=DEV)
    ys = [blk.step(x[:, t], state) for t in range(9)]
    assert torch.allclose(y_full, torch.stack(ys, 1), atol=1e-5)


def test_pathway_block_grads_match_autograd():
    blk = make_pathway_block()
    x = torch.randn(2, 12, 16, device=DEV)
    blk(x).pow(2).sum().backward()
    params = {k: v.detach().double().cpu().requires_grad_() for k, v in blk.state_dict().items()}

    def scan(xc, delta, A, B, C, Dv):
        hst = torch.zeros(xc.shape[0], xc.shape[2], A.shape[1], dtype=torch.float64)
        ys = []
        for t in range(xc.shape[1]):
            hst = torch.exp(delta[:, t, :, None] * A) * hst + delta[:, t, :, None] * B[:, t, None, :] * xc[:, t, :, None]
            ys.append((hst * C[:, t, None, :]).sum(-1))
        return torch.stack(ys, 1) + xc * Dv

    # the block of _pathway_reference again, on grad-tracking float64 copies of the parameters
    h = x.double().cpu()
    p = params
    xz = h @ p["in_proj.weight"].T
    D = blk.d_inner
    xx, z = xz[..., :D], xz[..., D:]
    L = xx.shape[1]
    xc = F.silu(F.conv1d(xx.transpose(1, 2), p["conv1d.weight"], p["conv1d.bias"], padding=3,
                         groups=D)[..., :L].transpose(1, 2))
    dt, B, C = torch.split(xc @ p["x_proj.weight"].T, [blk.dt_rank, blk.d_state, blk.d_state], dim=-1)
    delta = F.softplus(dt @ p["dt_proj.weight"].T + p["dt_proj.bias"])
    y = scan(xc, delta, -torch.exp(p["A_log"]), B, C, p["D"])
    w = torch.softmax(xc @ p["pathway.weight"].T + p["pathway.bias"], dim=-1) * blk.n_groups
    y = y * w[..., blk.group_of.cpu()] * F.silu(z)
    (y @ p["out_proj.weight"].T).pow(2).sum().backward()
    got = dict(blk.named_parameters())
    assert "pathway.weight" in got and "pathway.bias" in got
    for k, v in p.items():
        np.testing.assert_allclose(got[k].grad.double().cpu().numpy(), v.grad.numpy(), rtol=1e-3, atol=1e-4,
                                   err_msg=k)


def test_pathway_block_matches_reference_fixture(golden):
    """The reference's own SiftX block (pathway.npz, made by importing models/sift_block.py):
    its weights loaded into this block give the same forward output and recurrent steps."""
    g = golden("pathway")
    blk = SiftBlock(d_model=16, d_state=8, d_conv=4, expand=2,
                    timescales=[(1e-3, 1e-2), (1e-2, 3e-2), (3e-2, 1e-1)], pathway_gate=True).to(DEV)
    sd = {k[2:].replace("__", "."): torch.from_numpy(v).float() for k, v in g.items() if k.startswith("p_")}
    blk.load_state_dict(sd)
    assert blk.group_of.cpu().tolist() == g["group_of"].tolist()
    hidden = torch.from_numpy(g["hidden"]).float().to(DEV)
    scale = np.abs(g["out"]).max()
    np.testing.assert_allclose(blk(hidden).detach().double().cpu().numpy(), g["out"], rtol=1e-4, atol=1e-5 * scale)
    state = blk.allocate_state(2, device=DEV)
    steps = torch.stack([blk.step(hidden[:, t], state) for t in range(9)], 1)
    np.testing.assert_allclose(steps.detach().double().cpu().numpy(), g["steps"], rtol=1e-4, atol=1e-5 * scale)


def test_graphed_step_matches_eager_step():
    """GraphedStep replays SiftLM.step from one CUDA graph: the same logits token by token
    and the same state, and generate(graphed=True) picks the same greedy tokens."""
    from swiftx_b200.sift import GraphedStep
    torch.manual_seed(0)
    m = SiftLM(tiny_cfg()).to(DEV).eval()
    idx = torch.randint(0, 11, (3, 10), device=DEV)
    state = m.allocate_state(3, device=DEV)
    gs = GraphedStep(m, 3)
    for t in range(10):
        want = m.step(idx[:, t], state)
        got = gs(idx[:, t])
        assert torch.allclose(got, want, atol=1e-5, rtol=1e-5)
    for (c1, s1), (c2, s2) in zip(state, gs.state):
        assert torch.allclose(c1, c2, atol=1e-6) and torch.allclose(s1, s2, atol=1e-5)
    gs.reset()
    assert all(float(c.abs().sum()) == 0 and float(s.abs().sum()) == 0 for c, s in gs.state)
    a = m.generate(idx[:, :4], 6, temperature=0)
    b = m.generate(idx[:, :4], 6, temperature=0, graphed=True)
    assert torch.equal(a, b)


def test_graphed_step_bf16_weight_copies():
    """GraphedStep under bf16 autocast reads bf16 copies of the projection weights taken
    when it was built: its logits agree with the eager step under autocast (which casts
    every weight at every call) to bf16 rounding, go stale once a weight changes, and
    agree again after refresh_weights()."""
    from swiftx_b200.sift import GraphedStep
    torch.manual_seed(0)
    m = SiftLM(tiny_cfg()).to(DEV).eval()
    idx = torch.randint(0, 11, (3, 6), device=DEV)

    def eager():
        st = m.allocate_state(3, device=DEV)
        with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
            return torch.stack([m.step(idx[:, t], st).float() for t in range(6)])

    def graphed(gs):
        gs.reset()
        return torch.stack([gs(idx[:, t]).float().clone() for t in range(6)])

    def rel(a, b):
        return float((a - b).abs().max() / b.abs().max())

    gs = GraphedStep(m, 3, autocast_dtype=torch.bfloat16)
    assert gs._w16_flat is not None
    assert rel(graphed(gs), eager()) < 1e-2
    with torch.no_grad():
        for layer in m.backbone.layers:
            layer.mixer.out_proj.weight.mul_(10.0)
    want = eager()
    assert rel(graphed(gs), want) > 0.1            # the copies are from before the change
    gs.refresh_weights()
    assert rel(graphed(gs), want) < 1e-2
