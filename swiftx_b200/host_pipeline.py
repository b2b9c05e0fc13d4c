"""Forward + backward selective scan of host-resident batches, streamed through one GPU.

The reference runs its scan on whatever device the tensors live on
(models/selective_scan.py:246-265); a caller whose batches sit in host memory pays for
the copies.  This executor keeps them off the critical path: the batch rows are cut
into chunks, and every chunk goes

    H2D (copy stream) -> forward + backward kernels (compute stream) -> D2H (copy stream)

(the forward starts once u, delta, z, B, C are in, while dout is still on its way, and
the output's copy out starts as soon as the forward ends)

over ``nbuf`` rotating sets of device buffers, so that the copy of chunk k+1 in, the
kernels of chunk k and the copy of chunk k-1 out run at the same time.  PCIe is full
duplex and the two copy directions use separate copy engines, so a step costs about
the larger of the two transfers plus one chunk's kernels, not the sum of everything.
Chunks of a few rows leave most SMs idle, so consecutive chunks alternate between
``n_compute`` compute streams and their kernels overlap too.

The batch rows of the scan are independent (models/selective_scan.py:34-60 loops over
time only), so chunking by rows changes no value: out, du, ddelta, dz, dB, dC of a row
are what the whole-batch call gives.  dA, dD and d(delta_bias) -- sums over the batch
-- are kept per chunk on the device and added in chunk order at the end (deterministic,
and equal to the whole-batch kernel's fixed-order sum up to fp32 reassociation).

Host tensors must be pinned (``tensor.pin_memory()``) for the copies to overlap;
pageable memory works but serialises the copies.
"""
import torch

from . import _lib
# fp32 or bf16 rows; parameters, partial sums, checkpoints and the pre-gate output are
# fp32 buffers sized for these two (the float64 kernels take float64 throughout)
_ROW_DTYPES = (torch.float32, torch.bfloat16)

_INPUTS = ("u", "delta", "z", "B", "C", "dout")
_ROW_GRADS = ("du", "ddelta", "dz", "dB", "dC")


class HostScanPipeline:
    """Preallocated device buffers and streams for one problem shape.

    batch, seqlen, dim, dstate: the (b, L, D, N) of every call; dtype: float32 or
    bfloat16 for u, delta, z, B, C, dout and the row gradients; has_z / has_D /
    has_bias: which optional operands the calls pass.

    chain_calls: when False (default) every call is queued behind the current stream,
    as a torch copy would be.  When True, a call's copies in wait only for this
    pipeline's own earlier work, so the next call's inputs stream in while the previous
    call's last kernels and copies out finish (a loader feeding one batch after the
    other); the host inputs must then be ready when the call is made, not produced by
    work still queued on the current stream.  Either way the current stream waits for
    the call's results."""

    def __init__(self, batch, seqlen, dim, dstate, *, dtype=torch.float32, has_z=True, has_D=True,
                 has_bias=True, delta_softplus=True, rows_per_chunk=None, nbuf=3, n_compute=2,
                 device=None, chain_calls=False):
        if dtype not in _ROW_DTYPES:
            raise ValueError(f"dtype must be float32 or bfloat16, got {dtype}")
        if not 1 <= dstate <= 16:
            raise ValueError(f"d_state must be in 1..16, got {dstate}")
        self.lib = _lib.load()
        dev = torch.device(device if device is not None else "cuda")
        if dev.type == "cuda" and dev.index is None:
            dev = torch.device("cuda", torch.cuda.current_device())
        self.dev = dev
        if dev.type != "cuda":
            raise RuntimeError("HostScanPipeline needs a CUDA device (no CPU path)")
        self.b, self.L, self.D, self.N = batch, seqlen, dim, dstate
        self.dtype, self.has_z, self.has_D, self.has_bias = dtype, has_z, has_D, has_bias
        self.softplus = bool(delta_softplus)
        self.rows = rows_per_chunk or max(1, -(-batch // 8))
        self.chunks = [(r, min(batch, r + self.rows)) for r in range(0, batch, self.rows)]
        # buffer sets beyond the chunk count only help when calls overlap one another
        self.nbuf = max(1, nbuf if chain_calls else min(nbuf, len(self.chunks)))
        self.n_compute = max(1, min(n_compute, self.nbuf))
        R, L, D, N, dev = self.rows, seqlen, dim, dstate, self.dev
        e = lambda *s, dt=dtype: torch.empty(s, device=dev, dtype=dt)  # noqa: E731
        ck_floats = self.lib.swx_scan_checkpoint_floats(R, L, D)
        self.ws_bytes = self.lib.swx_scan_bwd_workspace_bytes(R, L, D)
        self.sets = []
        for _ in range(self.nbuf):
            s = {k: e(R, L, N if k in ("B", "C") else D) for k in _INPUTS if k != "z" or has_z}
            s.update({k: e(R, L, N if k in ("dB", "dC") else D) for k in _ROW_GRADS if k != "dz" or has_z})
            s["out"] = e(R, L, D)
            s["pre"] = e(R, L, D, dt=torch.float32) if has_z else None
            s["ck"] = e(max(ck_floats, 1), dt=torch.float32)
            s["ws"] = e(max(self.ws_bytes, 1), dt=torch.uint8)
            self.sets.append(s)
        nc = len(self.chunks)
        # Per-call state that a chained call may still be using while the next one starts
        # (parameters, per-chunk partials of the batch sums, the sums themselves): two
        # copies, alternated by call parity.
        self.par = []
        for _ in range(2):
            self.par.append({
                "A": e(D, N, dt=torch.float32),
                "Dv": e(D, dt=torch.float32) if has_D else None,
                "bias": e(D, dt=torch.float32) if has_bias else None,
                "dA_part": e(nc, D, N, dt=torch.float32),
                "dD_part": e(nc, D, dt=torch.float32) if has_D else None,
                "dbias_part": e(nc, D, dt=torch.float32) if has_bias else None,
                "dA": e(D, N, dt=torch.float32),
                "dD": e(D, dt=torch.float32) if has_D else None,
                "dbias": e(D, dt=torch.float32) if has_bias else None,
                "ev_params": torch.cuda.Event(),   # parameters on the device
                "ev_done": None,                   # the call's last copy out finished
            })
        self.calls = 0
        self.turn = 0                              # chunks issued so far, over all calls
        self.chain_calls = bool(chain_calls)
        self.h2d = torch.cuda.Stream(dev)
        self.d2h = torch.cuda.Stream(dev)
        self.comp = [torch.cuda.Stream(dev) for _ in range(self.n_compute)]
        # per buffer set, re-recorded at every use (a wait sees the latest record)
        self.ev_in_free = [None] * self.nbuf      # set's inputs no longer read (kernels done)
        self.ev_out_free = [None] * self.nbuf     # set's results copied out
        self.ev_in_fwd = [torch.cuda.Event() for _ in range(self.nbuf)]   # forward inputs in
        self.ev_in = [torch.cuda.Event() for _ in range(self.nbuf)]       # all inputs in
        self.ev_fwd = [torch.cuda.Event() for _ in range(self.nbuf)]      # forward done

    # ------------------------------------------------------------------ host buffers
    def allocate_host_outputs(self):
        """Pinned host tensors for every result of ``forward_backward``."""
        b, L, D, N = self.b, self.L, self.D, self.N
        p = lambda *s, dt=self.dtype: torch.empty(s, dtype=dt).pin_memory()  # noqa: E731
        out = {"out": p(b, L, D), "du": p(b, L, D), "ddelta": p(b, L, D), "dB": p(b, L, N), "dC": p(b, L, N),
               "dA": p(D, N, dt=torch.float32)}
        if self.has_z:
            out["dz"] = p(b, L, D)
        if self.has_D:
            out["dD"] = p(D, dt=torch.float32)
        if self.has_bias:
            out["ddelta_bias"] = p(D, dt=torch.float32)
        return out

    def _check_host(self, name, t, shape, dtype):
        if t is None:
            raise ValueError(f"{name} is required by this pipeline")
        if t.device.type != "cpu":
            raise ValueError(f"{name} must be a host tensor")
        if tuple(t.shape) != shape or t.dtype != dtype or not t.is_contiguous():
            raise ValueError(f"{name}: expected contiguous {dtype} {shape}, got {t.dtype} {tuple(t.shape)}")

    # ------------------------------------------------------------------ one step
    def _args(self, s, pr, rows, fwd):
        """swx_scan_args over the device buffers of set `s` (parameters from `pr`) for a
        chunk of `rows` rows."""
        a = _lib.ScanArgs()
        a.batch, a.seqlen, a.dim, a.dstate = rows, self.L, self.D, self.N
        a.in_dtype = a.out_dtype = _lib.DTYPE_CODES[self.dtype]
        a.delta_softplus = 1 if self.softplus else 0
        L, D, N = self.L, self.D, self.N
        a.u, a.u_sb, a.u_sl = s["u"].data_ptr(), L * D, D
        a.delta, a.delta_sb, a.delta_sl = s["delta"].data_ptr(), L * D, D
        if self.has_z:
            a.z, a.z_sb, a.z_sl = s["z"].data_ptr(), L * D, D
            a.out_pre = s["pre"].data_ptr()
        a.B, a.B_sb, a.B_sl = s["B"].data_ptr(), L * N, N
        a.C, a.C_sb, a.C_sl = s["C"].data_ptr(), L * N, N
        a.A = pr["A"].data_ptr()
        a.Dskip = pr["Dv"].data_ptr() if self.has_D else None
        a.delta_bias = pr["bias"].data_ptr() if self.has_bias else None
        a.checkpoints = s["ck"].data_ptr()
        if fwd:
            a.out = s["out"].data_ptr()
        else:
            a.dout, a.dout_sb, a.dout_sl = s["dout"].data_ptr(), L * D, D
            for k in _ROW_GRADS:
                if k in s:
                    setattr(a, k, s[k].data_ptr())
            a.workspace, a.workspace_bytes = s["ws"].data_ptr(), self.ws_bytes
        return a

    def forward_backward(self, u, delta, A, B, C, dout, D=None, z=None, delta_bias=None, out=None):
        """out = selective_scan_fn(u, delta, A, B, C, D, z, delta_bias, softplus) and its
        gradients for the upstream gradient ``dout``, all on host tensors.

        Returns a dict of pinned host tensors (``out``, ``du``, ``ddelta``, ``dz``, ``dB``,
        ``dC``, ``dA``, ``dD``, ``ddelta_bias``); pass ``out`` (from
        ``allocate_host_outputs``) to reuse buffers.  The work is queued behind the
        current stream and the current stream waits for it; synchronize before reading
        the results on the host."""
        b, L, Dm, N = self.b, self.L, self.D, self.N
        dt = self.dtype
        for name, t, shp in (("u", u, (b, L, Dm)), ("delta", delta, (b, L, Dm)), ("B", B, (b, L, N)),
                             ("C", C, (b, L, N)), ("dout", dout, (b, L, Dm))):
            self._check_host(name, t, shp, dt)
        if self.has_z:
            self._check_host("z", z, (b, L, Dm), dt)
        elif z is not None:
            raise ValueError("this pipeline was built without z")
        self._check_host("A", A, (Dm, N), torch.float32)
        if self.has_D:
            self._check_host("D", D, (Dm,), torch.float32)
        if self.has_bias:
            self._check_host("delta_bias", delta_bias, (Dm,), torch.float32)
        res = out if out is not None else self.allocate_host_outputs()
        host_in = {"u": u, "delta": delta, "z": z, "B": B, "C": C, "dout": dout}
        lib, main = self.lib, torch.cuda.current_stream(self.dev)
        pr = self.par[self.calls % 2]
        self.calls += 1

        if not self.chain_calls:
            self.h2d.wait_stream(main)
            self.d2h.wait_stream(main)
            for cs in self.comp:
                cs.wait_stream(main)
        with torch.cuda.stream(self.h2d):
            if pr["ev_done"] is not None:                 # the call two back is finished with pr
                self.h2d.wait_event(pr["ev_done"])
            pr["A"].copy_(A, non_blocking=True)
            if self.has_D:
                pr["Dv"].copy_(D, non_blocking=True)
            if self.has_bias:
                pr["bias"].copy_(delta_bias, non_blocking=True)
            pr["ev_params"].record(self.h2d)
        for cs in self.comp:
            cs.wait_event(pr["ev_params"])

        for k, (r0, r1) in enumerate(self.chunks):
            n = r1 - r0
            si = self.turn % self.nbuf
            s = self.sets[si]
            cs = self.comp[self.turn % self.n_compute]
            self.turn += 1
            with torch.cuda.stream(self.h2d):
                if self.ev_in_free[si] is not None:
                    self.h2d.wait_event(self.ev_in_free[si])     # set's inputs no longer read
                for name in _INPUTS:
                    if name == "dout":                 # the forward need not wait for it
                        self.ev_in_fwd[si].record(self.h2d)
                    if name in s:
                        s[name][:n].copy_(host_in[name][r0:r1], non_blocking=True)
                self.ev_in[si].record(self.h2d)
            cs.wait_event(self.ev_in_fwd[si])
            if self.ev_out_free[si] is not None:
                cs.wait_event(self.ev_out_free[si])              # set's results copied out
            sp = _lib.vp(cs.cuda_stream)
            _lib.check(lib.swx_scan_fwd(self._args(s, pr, n, True), sp), "swx_scan_fwd")
            self.ev_fwd[si].record(cs)
            with torch.cuda.stream(self.d2h):          # the output leaves while the backward runs
                self.d2h.wait_event(self.ev_fwd[si])
                res["out"][r0:r1].copy_(s["out"][:n], non_blocking=True)
            cs.wait_event(self.ev_in[si])
            a = self._args(s, pr, n, False)
            a.dA = pr["dA_part"][k].data_ptr()
            a.dD = pr["dD_part"][k].data_ptr() if self.has_D else None
            a.ddelta_bias = pr["dbias_part"][k].data_ptr() if self.has_bias else None
            _lib.check(lib.swx_scan_bwd(a, sp), "swx_scan_bwd")
            self.ev_in_free[si] = cs.record_event()
            with torch.cuda.stream(self.d2h):
                self.d2h.wait_event(self.ev_in_free[si])
                for name in _ROW_GRADS:
                    if name in s:
                        res[name][r0:r1].copy_(s[name][:n], non_blocking=True)
                self.ev_out_free[si] = self.d2h.record_event()

        # batch-summed gradients: chunk partials added in chunk order, then one copy out
        c0 = self.comp[0]
        for cs in self.comp[1:]:
            c0.wait_stream(cs)
        with torch.cuda.stream(c0):
            torch.sum(pr["dA_part"], 0, out=pr["dA"])
            if self.has_D:
                torch.sum(pr["dD_part"], 0, out=pr["dD"])
            if self.has_bias:
                torch.sum(pr["dbias_part"], 0, out=pr["dbias"])
        with torch.cuda.stream(self.d2h):
            self.d2h.wait_stream(c0)
            res["dA"].copy_(pr["dA"], non_blocking=True)
            if self.has_D:
                res["dD"].copy_(pr["dD"], non_blocking=True)
            if self.has_bias:
                res["ddelta_bias"].copy_(pr["dbias"], non_blocking=True)
            pr["ev_done"] = self.d2h.record_event()
        main.wait_stream(self.d2h)
        main.wait_stream(self.h2d)
        return res

    @staticmethod
    def d2h_bytes(res):
        return sum(t.numel() * t.element_size() for t in res.values())
