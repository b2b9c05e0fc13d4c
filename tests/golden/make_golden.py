"""Generate golden vectors for the selective-scan path from the reference itself.

Run once, in a container where the reference project is checked out (read-only):

    python tests/golden/make_golden.py /path/to/reference

It imports the reference's own Python modules (models.selective_scan,
models.sift_block) and records inputs and outputs as small .npz fixtures in this
folder.  The fixtures travel with the repository; the reference does not.

Fixtures:
  hand_tiny.npz      tests/test_selective_scan.py:31-40 known answer (y = [2, 5, 8.5])
  fwd_L{1,7,64}.npz  tests/test_selective_scan.py:68-74 shapes (b=2, D=8, N=16, seed 1)
  bwd_f64.npz        tests/test_selective_scan.py:77-86 shapes (float64, b=2, L=20, D=5, N=6, seed 2)
  tail_*.npz         tests/test_triton_scan.py:15 tail shapes, forward + all grads
  fwd_b2_L256_D128.npz  b=2, L=256, D=128, N=16, seed 0, forward only (the CPU-sized case)
  gated.npz          scan(u, softplus(dr + bias)) * silu(z) via the block's glue, all grads
  conv.npz           SiftBlock conv1d + SiLU on the strided x half of in_proj, with grads
  decode.npz         SiftBlock.step intermediates (conv window, state update, gated y)
  pathway.npz        SiftX block (3 timescale groups, pathway gate): weights, forward output
                     and 9 recurrent steps (models/sift_block.py:111-175)
  linscan.npz        parallel_scan / sequential_scan on tests/test_selective_scan.py:59-64
                     shapes, and float64 gradients of sequential_scan by autograd

    python tests/golden/make_golden.py /path/to/reference --only pathway

regenerates one fixture.
"""
import math
import os
import sys

import numpy as np
import torch
import torch.nn.functional as F

HERE = os.path.dirname(os.path.abspath(__file__))


def save(name, **arrs):
    out = {k: (v.detach().cpu().numpy() if torch.is_tensor(v) else np.asarray(v))
           for k, v in arrs.items() if v is not None}
    np.savez_compressed(os.path.join(HERE, name + ".npz"), **out)
    print("wrote", name, {k: v.shape for k, v in out.items()})


def make_inputs(b, L, D, N, seed, dtype=torch.float32):
    """Same generator as the reference test suite (tests/test_selective_scan.py:14-22)."""
    g = torch.Generator().manual_seed(seed)
    u = torch.randn(b, L, D, generator=g)
    delta = torch.rand(b, L, D, generator=g) * 0.5 + 0.01
    A = -torch.rand(D, N, generator=g) - 0.1
    B = torch.randn(b, L, N, generator=g)
    C = torch.randn(b, L, N, generator=g)
    Dskip = torch.randn(D, generator=g)
    return [t.to(dtype) for t in (u, delta, A, B, C, Dskip)]


def config_inputs(b, L, D, N, seed=0):
    """The benchmark value distributions: u ~ N(0,1); delta_raw ~ N(0,0.5); bias =
    inverse-softplus(dt), dt log-uniform in [1e-3, 0.1]; A = -(1..N); B, C ~ N(0,1);
    D = 1; z ~ N(0,1).  Drawn in (b, D, L) / (b, N, L) order, then transposed to the
    reference layout (b, L, D) / (b, L, N)."""
    g = torch.Generator().manual_seed(seed)
    u = torch.randn(b, D, L, generator=g).transpose(1, 2).contiguous()
    dr = (torch.randn(b, D, L, generator=g) * 0.5).transpose(1, 2).contiguous()
    dt = torch.exp(torch.rand(D, generator=g) * (math.log(0.1) - math.log(1e-3)) + math.log(1e-3))
    bias = dt + torch.log(-torch.expm1(-dt))
    A = -torch.arange(1, N + 1, dtype=torch.float32).repeat(D, 1)
    Bm = torch.randn(b, N, L, generator=g).transpose(1, 2).contiguous()
    Cm = torch.randn(b, N, L, generator=g).transpose(1, 2).contiguous()
    Dskip = torch.ones(D)
    z = torch.randn(b, D, L, generator=g).transpose(1, 2).contiguous()
    return u, dr, bias, A, Bm, Cm, Dskip, z


def make_pathway(SiftBlock):
    """9. SiftX block with pathway mixing (models/sift_block.py:74-93, 111-142, 153-175)."""
    torch.manual_seed(0)
    blk = SiftBlock(d_model=16, d_state=8, d_conv=4, expand=2, scan_impl="ref",
                    timescales=[(1e-3, 1e-2), (1e-2, 3e-2), (3e-2, 1e-1)], pathway_gate=True).double()
    gen = torch.Generator().manual_seed(11)
    with torch.no_grad():
        blk.pathway.weight.copy_(0.5 * torch.randn(blk.pathway.weight.shape, dtype=torch.float64, generator=gen))
        blk.pathway.bias.copy_(0.5 * torch.randn(blk.pathway.bias.shape, dtype=torch.float64, generator=gen))
        hidden = torch.randn(2, 29, 16, dtype=torch.float64, generator=gen)
        out = blk(hidden)
        state = blk.allocate_state(2, dtype=torch.float64)
        steps = torch.stack([blk.step(hidden[:, t], state) for t in range(9)], 1)
    params = {"p_" + k.replace(".", "__"): v for k, v in blk.state_dict().items()}
    save("pathway", hidden=hidden, out=out, steps=steps, group_of=blk.group_of, **params)


def make_linscan(parallel_scan, sequential_scan):
    """10. The associative and the loop scan (models/selective_scan.py:66-99) on the
    reference test's inputs (tests/test_selective_scan.py:59-64), plus float64 gradients by
    autograd through sequential_scan."""
    out = {}
    for L in (1, 2, 5, 8, 33, 128):
        g = torch.Generator().manual_seed(L)
        a = torch.rand(3, L, 4, 2, generator=g)
        x = torch.randn(3, L, 4, 2, generator=g)
        out.update({f"a_{L}": a, f"x_{L}": x, f"hp_{L}": parallel_scan(a, x), f"hs_{L}": sequential_scan(a, x)})
    g = torch.Generator().manual_seed(99)
    a = torch.rand(2, 33, 5, 3, dtype=torch.float64, generator=g).requires_grad_()
    x = torch.randn(2, 33, 5, 3, dtype=torch.float64, generator=g).requires_grad_()
    w = torch.randn(2, 33, 5, 3, dtype=torch.float64, generator=g)
    h = sequential_scan(a, x)         # parallel_scan's in-place updates are not differentiable
    (h * w).sum().backward()
    out.update(ga=a.detach(), gx=x.detach(), gw=w, gh=h.detach(), gda=a.grad, gdx=x.grad)
    save("linscan", **out)


def main(ref_root, only=None):
    sys.path.insert(0, ref_root)
    from models.selective_scan import selective_scan_fast, selective_scan_ref
    from models.sift_block import SiftBlock
    if only == "pathway":
        make_pathway(SiftBlock)
        return
    if only == "linscan":
        from models.selective_scan import parallel_scan, sequential_scan
        make_linscan(parallel_scan, sequential_scan)
        return

    # 1. hand-computed known answer
    u = torch.tensor([[[2.0], [4.0], [6.0]]])
    delta = torch.ones(1, 3, 1)
    A = torch.tensor([[-math.log(2.0)]])
    Bm = torch.ones(1, 3, 1)
    Cm = torch.ones(1, 3, 1)
    save("hand_tiny", u=u, delta=delta, A=A, B=Bm, C=Cm, y=selective_scan_ref(u, delta, A, Bm, Cm))

    # 2. forward shapes of the reference fast-vs-ref test
    for L in (1, 7, 64):
        u, dl, A, Bm, Cm, Ds = make_inputs(2, L, 8, 16, 1)
        y = selective_scan_ref(*(t.double() for t in (u, dl, A, Bm, Cm, Ds)))
        save(f"fwd_L{L}", u=u, delta=dl, A=A, B=Bm, C=Cm, D=Ds, y=y)

    # 3. float64 backward of the reference
    ins = make_inputs(2, 20, 5, 6, 2, dtype=torch.float64)
    a = [t.clone().requires_grad_() for t in ins]
    gy = torch.randn(2, 20, 5, dtype=torch.float64, generator=torch.Generator().manual_seed(3))
    y = selective_scan_ref(*a)
    (y * gy).sum().backward()
    save("bwd_f64", u=ins[0], delta=ins[1], A=ins[2], B=ins[3], C=ins[4], D=ins[5], gy=gy, y=y,
         du=a[0].grad, ddelta=a[1].grad, dA=a[2].grad, dB=a[3].grad, dC=a[4].grad, dD=a[5].grad)

    # 4. tail shapes of the reference Triton test (non-power-of-2 D/N, L not a multiple of chunk)
    g = torch.Generator().manual_seed(0)
    for (b, L, D, N, K, hasD) in [(2, 37, 40, 16, 8, True), (1, 20, 8, 5, 64, False)]:
        u = torch.randn(b, L, D, generator=g, dtype=torch.float64)
        dl = torch.rand(b, L, D, generator=g, dtype=torch.float64) * 0.2 + 0.01
        A = -torch.rand(D, N, generator=g, dtype=torch.float64) - 0.5
        Bm = torch.randn(b, L, N, generator=g, dtype=torch.float64)
        Cm = torch.randn(b, L, N, generator=g, dtype=torch.float64)
        Dp = torch.randn(D, generator=g, dtype=torch.float64) if hasD else None
        gy = torch.randn(b, L, D, generator=g, dtype=torch.float64)
        ins = [t.float().double().requires_grad_() for t in (u, dl, A, Bm, Cm)]
        Dq = Dp.float().double().requires_grad_() if hasD else None
        y = selective_scan_ref(*ins, Dq)
        grads = torch.autograd.grad(y, ins + ([Dq] if hasD else []), gy.float().double())
        names = ["du", "ddelta", "dA", "dB", "dC"] + (["dD"] if hasD else [])
        save(f"tail_{b}x{L}x{D}x{N}", u=ins[0].float(), delta=ins[1].float(), A=ins[2].float(),
             B=ins[3].float(), C=ins[4].float(), D=(Dq.float() if hasD else None), gy=gy.float(),
             y=y, **dict(zip(names, grads)))

    # 5. the CPU config (forward only, no gate): fp32 inputs, fp64 reference output,
    #    and the reference's fused CPU path in fp32 for comparison
    u, dr, bias, A, Bm, Cm, Ds, _ = config_inputs(2, 256, 128, 16, seed=0)
    delta = F.softplus(dr + bias)
    y64 = selective_scan_ref(u.double(), delta.double(), A.double(), Bm.double(), Cm.double(), Ds.double())
    y32 = selective_scan_fast(u, delta, A, Bm, Cm, Ds, mode="fused")
    save("fwd_b2_L256_D128", u=u, delta_raw=dr, delta_bias=bias, delta=delta, A=A, B=Bm, C=Cm, D=Ds, y=y64,
         y_fused_f32=y32)

    # 6. gated scan with softplus(delta_raw + bias): the block's glue around the reference scan
    u, dr, bias, A, Bm, Cm, Ds, z = config_inputs(2, 33, 24, 16, seed=5)
    Ds = Ds + 0.25 * torch.randn(24, generator=torch.Generator().manual_seed(6))
    leaves = [t.double().requires_grad_() for t in (u, dr, bias, A, Bm, Cm, Ds, z)]
    uu, drr, bb, AA, BB, CC, DD, zz = leaves
    out = selective_scan_ref(uu, F.softplus(drr + bb), AA, BB, CC, DD) * F.silu(zz)
    gout = torch.randn(out.shape, dtype=torch.float64, generator=torch.Generator().manual_seed(7))
    grads = torch.autograd.grad(out, leaves, gout)
    save("gated", u=u, delta_raw=dr, delta_bias=bias, A=A, B=Bm, C=Cm, D=Ds, z=z, gout=gout, out=out,
         du=grads[0], ddelta=grads[1], ddelta_bias=grads[2], dA=grads[3], dB=grads[4], dC=grads[5],
         dD=grads[6], dz=grads[7])

    # 7. conv1d + SiLU of the block, on the strided x half of the in_proj output
    torch.manual_seed(0)
    blk = SiftBlock(d_model=16, d_state=8, d_conv=4, expand=2).double()
    hidden = torch.randn(2, 13, 16, dtype=torch.float64)
    xz = blk.in_proj(hidden).detach().requires_grad_()
    x, _ = xz.chunk(2, dim=-1)
    L = x.shape[1]
    xc = F.silu(blk.conv1d(x.transpose(1, 2))[..., :L].transpose(1, 2))
    gc = torch.randn(xc.shape, dtype=torch.float64, generator=torch.Generator().manual_seed(8))
    dxz, dw, db = torch.autograd.grad(xc, [xz, blk.conv1d.weight, blk.conv1d.bias], gc)
    save("conv", xz=xz, w=blk.conv1d.weight.squeeze(1), bias=blk.conv1d.bias, out=xc, gout=gc,
         dx=dxz[..., :xz.shape[-1] // 2], dw=dw.squeeze(1), dbias=db)

    # 8. decode step intermediates of SiftBlock.step (models/sift_block.py:153-175)
    torch.manual_seed(0)
    blk = SiftBlock(d_model=16, d_state=8, d_conv=4, expand=2).double()
    state = blk.allocate_state(3, dtype=torch.float64)
    gen = torch.Generator().manual_seed(9)
    state[0].copy_(torch.randn(state[0].shape, dtype=torch.float64, generator=gen))
    state[1].copy_(0.1 * torch.randn(state[1].shape, dtype=torch.float64, generator=gen))
    conv0, ssm0 = state[0].clone(), state[1].clone()
    cap = {}
    dt_fwd, out_fwd, in_fwd = blk.dt_proj.forward, blk.out_proj.forward, blk.in_proj.forward
    blk.in_proj.forward = lambda h: cap.setdefault("xz", in_fwd(h))
    blk.dt_proj.forward = lambda t: cap.setdefault("dr", dt_fwd(t))
    blk.out_proj.forward = lambda y: cap.setdefault("y", y)
    x_proj_fwd = blk.x_proj.forward
    blk.x_proj.forward = lambda t: cap.setdefault("xdbl", x_proj_fwd(t))
    hidden = torch.randn(3, 16, dtype=torch.float64, generator=gen)
    with torch.no_grad():
        blk.step(hidden, state)
    xz = cap["xz"]
    x, z = xz.chunk(2, dim=-1)
    _, Bm, Cm = torch.split(cap["xdbl"], [blk.dt_rank, blk.d_state, blk.d_state], dim=-1)
    save("decode", x=x, z=z, delta_raw=cap["dr"], B=Bm, C=Cm, conv_w=blk.conv1d.weight.squeeze(1),
         conv_b=blk.conv1d.bias, A=-torch.exp(blk.A_log.float()).double(), D=blk.D, conv_state0=conv0, ssm_state0=ssm0,
         y=cap["y"], conv_state1=state[0], ssm_state1=state[1])

    make_pathway(SiftBlock)
    from models.selective_scan import parallel_scan, sequential_scan
    make_linscan(parallel_scan, sequential_scan)


if __name__ == "__main__":
    args = [a for a in sys.argv[1:] if a != "--only"]
    only = sys.argv[sys.argv.index("--only") + 1] if "--only" in sys.argv else None
    if only:
        args.remove(only)
    ref = args[0] if args else os.environ.get("SWIFTX_REFERENCE")
    if not ref:
        sys.exit("usage: make_golden.py <path to the reference checkout> [--only NAME] "
                 "(or set SWIFTX_REFERENCE)")
    main(ref, only)
