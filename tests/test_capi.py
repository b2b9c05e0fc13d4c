"""The C-ABI library loads and exports every entry point include/swiftx_b200.h declares;
argument validation runs on the host before any CUDA call (no GPU needed)."""
import ctypes
import os
import re

import pytest

from swiftx_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    src = open(os.path.join(ROOT, "include", "swiftx_b200.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(swx_[a-z0-9_]+)\s*\(", src)))


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    names = declared_functions()
    assert len(names) >= 10
    for n in names:
        assert hasattr(lib, n), f"missing export {n}"


def test_struct_mirrors_match():
    lib = _lib.load()
    assert lib.swx_scan_args_size() == ctypes.sizeof(_lib.ScanArgs)
    assert lib.swx_conv_args_size() == ctypes.sizeof(_lib.ConvArgs)
    assert lib.swx_decode_args_size() == ctypes.sizeof(_lib.DecodeArgs)
    assert lib.swx_linear_scan_args_size() == ctypes.sizeof(_lib.LinearScanArgs)
    assert lib.swx_rmsnorm_args_size() == ctypes.sizeof(_lib.RMSNormArgs)
    assert lib.swx_embedding_args_size() == ctypes.sizeof(_lib.EmbeddingArgs)
    assert lib.swx_abi_version() == 13


def test_status_strings():
    lib = _lib.load()
    for code in range(5):
        assert lib.swx_status_string(code)
    assert lib.swx_status_string(0) == b"ok"


def test_sizes_of_checkpoints_and_workspace():
    lib = _lib.load()
    assert lib.swx_scan_checkpoint_floats(8, 2048, 512) == 8 * 128 * 512 * 16
    assert lib.swx_scan_checkpoint_floats(1, 17, 3) == 1 * 2 * 3 * 16
    # dB|dC partials per 64-channel block (8 x 8 rows x 2048 steps x 32 floats), plus the
    # per-segment partials, sub-segment summaries and segment carries
    def segments(b, L, D):                    # fp32 inputs: the segmented kernel, no device query
        a = _lib.ScanArgs()
        a.batch, a.seqlen, a.dim, a.dstate = b, L, D, 16
        a.in_dtype = a.out_dtype = 0
        a.u = a.delta = a.B = a.C = a.A = 256      # placeholders: the query reads no memory
        return lib.swx_scan_bwd_segments(ctypes.byref(a))
    nseg = segments(8, 2048, 512)
    assert nseg == 4 and segments(16, 512, 512) == 4 and segments(8, 64, 512) == 1
    assert segments(4, 65536, 2048) == 2 and segments(1, 65536, 2048) == 9 and segments(1, -1, 8) < 0
    assert segments(16, 2048, 512) == nseg                       # rows beyond 8 do not change the plan
    assert segments(1, 2048, 512) == 16                          # a single row: more segments
    ws = lib.swx_scan_bwd_workspace_bytes(8, 2048, 512)
    assert ws >= 8 * 8 * 2048 * 32 * 4 + nseg * 8 * 512 * (16 + 2) * 4 + (2048 // 128) * 8 * 512 * 17 * 4
    assert lib.swx_scan_bwd_workspace_bytes(65535, 1 << 30, 1 << 30) == -1
    assert lib.swx_scan_checkpoint_floats(-1, 4, 4) == -1
    assert lib.swx_scan_bwd_workspace_bytes_f64(8, 2048, 512) >= 16 * 8 * 2048 * 32 * 8
    # one (weight, bias) partial per (row, 16-step time tile, channel): 2 rows x 9 tiles x 8 ch x (4+1) floats
    assert lib.swx_conv1d_bwd_workspace_bytes(2, 130, 8, 4) == 2 * 9 * 8 * 5 * 4
    # one (vocab, dim) fp32 partial per token slice; slices hold >= 128 tokens
    assert lib.swx_embedding_bwd_workspace_bytes(0, 256, 256) == 0
    assert lib.swx_embedding_bwd_workspace_bytes(300, 10, 64) == 3 * 10 * 64 * 4
    assert lib.swx_embedding_bwd_workspace_bytes(-1, 10, 64) < 0


def test_host_side_validation_without_gpu():
    lib = _lib.load()
    # NULL argument block
    assert lib.swx_scan_fwd(None, None) == _lib.SWX_ERR_INVALID_ARG
    a = _lib.ScanArgs()
    a.batch, a.seqlen, a.dim, a.dstate = 1, 4, 4, 17          # N > 16
    assert lib.swx_scan_fwd(a, None) == _lib.SWX_ERR_UNSUPPORTED
    a.dstate, a.in_dtype = 16, 7                              # unknown dtype
    assert lib.swx_scan_fwd(a, None) == _lib.SWX_ERR_UNSUPPORTED
    a.in_dtype, a.flags = 0, 2                                # unknown flag bit
    assert lib.swx_scan_fwd(a, None) == _lib.SWX_ERR_INVALID_ARG
    a.flags = _lib.SWX_SCAN_A_LOG                             # missing pointers
    assert lib.swx_scan_fwd(a, None) == _lib.SWX_ERR_INVALID_ARG
    assert lib.swx_scan_bwd(a, None) == _lib.SWX_ERR_INVALID_ARG
    a.seqlen = 0                                              # empty problem: nothing to do
    assert lib.swx_scan_fwd(a, None) == _lib.SWX_OK
    a.batch, a.seqlen = 65536, 4                              # more rows than the grid's y dimension
    assert lib.swx_scan_fwd(a, None) == _lib.SWX_ERR_UNSUPPORTED
    assert lib.swx_scan_bwd(a, None) == _lib.SWX_ERR_UNSUPPORTED
    c = _lib.ConvArgs()
    c.batch, c.seqlen, c.dim, c.width = 1, 4, 4, 9            # width > 6
    assert lib.swx_conv1d_fwd(c, None) == _lib.SWX_ERR_UNSUPPORTED
    c.width, c.seqlen = 4, 65535 * 16 + 1                     # more time tiles than the grid's y dimension
    assert lib.swx_conv1d_fwd(c, None) == _lib.SWX_ERR_UNSUPPORTED
    d = _lib.DecodeArgs()
    d.batch, d.dim, d.mode = 1, 4, 0                          # no mode
    assert lib.swx_decode_step(d, None) == _lib.SWX_ERR_INVALID_ARG
    d.mode, d.flags = _lib.SWX_DECODE_SSM, 2                  # unknown flag bit
    assert lib.swx_decode_step(d, None) == _lib.SWX_ERR_INVALID_ARG
    s = _lib.LinearScanArgs()
    s.batch, s.seqlen, s.width, s.dtype = 2, 5, 3, 1          # bf16 is not a linear-scan dtype
    assert lib.swx_linear_scan_fwd(s, None) == _lib.SWX_ERR_UNSUPPORTED
    s.dtype = 0                                               # missing pointers
    assert lib.swx_linear_scan_fwd(s, None) == _lib.SWX_ERR_INVALID_ARG
    assert lib.swx_linear_scan_bwd(s, None) == _lib.SWX_ERR_INVALID_ARG
    s.seqlen = 0
    assert lib.swx_linear_scan_fwd(s, None) == _lib.SWX_OK
    r = _lib.RMSNormArgs()
    r.rows, r.dim, r.eps, r.dtype = 4, 2048, 1e-5, 0           # dim > 1024
    assert lib.swx_rmsnorm_fwd(r, None) == _lib.SWX_ERR_UNSUPPORTED
    r.dim = 256                                               # missing pointers
    assert lib.swx_rmsnorm_fwd(r, None) == _lib.SWX_ERR_INVALID_ARG
    assert lib.swx_rmsnorm_bwd(r, None) == _lib.SWX_ERR_INVALID_ARG
    r.residual, r.res_dtype = 1, 7                            # residual form: unknown residual dtype
    assert lib.swx_rmsnorm_fwd(r, None) == _lib.SWX_ERR_UNSUPPORTED
    r.res_dtype = 1                                           # residual without a sum output
    r.x, r.weight, r.y = 8, 8, 8
    assert lib.swx_rmsnorm_fwd(r, None) == _lib.SWX_ERR_INVALID_ARG
    r.residual = r.x = r.weight = r.y = None
    e = _lib.EmbeddingArgs()
    e.ntok, e.vocab, e.dim = 8, 2000, 32                      # vocab > 1024
    assert lib.swx_embedding_bwd(e, None) == _lib.SWX_ERR_UNSUPPORTED
    e.vocab = 256                                             # missing pointers
    assert lib.swx_embedding_bwd(e, None) == _lib.SWX_ERR_INVALID_ARG
    e.vocab = 0                                               # empty weight: nothing to do
    assert lib.swx_embedding_bwd(e, None) == _lib.SWX_OK


def test_cpu_tensors_are_rejected_not_computed():
    torch = pytest.importorskip("torch")
    from swiftx_b200 import selective_scan_fast
    from swiftx_b200.conv import causal_conv1d_fn
    u = torch.randn(1, 4, 3)
    with pytest.raises(RuntimeError):
        selective_scan_fast(u, u.abs(), -torch.ones(3, 2), torch.randn(1, 4, 2), torch.randn(1, 4, 2))
    with pytest.raises(RuntimeError):
        causal_conv1d_fn(u, torch.randn(3, 1, 4))
    from swiftx_b200 import parallel_scan
    with pytest.raises(RuntimeError):
        parallel_scan(torch.rand(2, 5, 3), torch.randn(2, 5, 3))
    from swiftx_b200.decode import decode_conv_step
    with pytest.raises(RuntimeError):
        decode_conv_step(torch.randn(2, 3), torch.zeros(2, 3, 4), torch.randn(3, 4))
    from swiftx_b200.norm import rms_norm
    with pytest.raises(ValueError):
        rms_norm(u, torch.ones(3))
    from swiftx_b200.host_pipeline import HostScanPipeline
    with pytest.raises(RuntimeError):
        HostScanPipeline(2, 8, 3, 2, device="cpu")
    for bad in (dict(dtype=torch.float64), dict(dstate=0), dict(dstate=17)):    # checked before any device use
        kw = dict(dtype=torch.float32, dstate=2) | bad
        with pytest.raises(ValueError):
            HostScanPipeline(2, 8, 3, kw.pop("dstate"), **kw)


def test_strided_gradient_output_arguments_are_checked():
    """dz / dx strides come in pairs and may not overlap rows; float64 takes dense dz only.
    The checks run before any device work."""
    lib = _lib.load()
    a = _lib.ScanArgs()
    a.batch, a.seqlen, a.dim, a.dstate = 2, 32, 64, 16
    a.in_dtype = a.out_dtype = 0                             # fp32
    for k in ("u", "delta", "B", "C", "A", "dout", "du", "ddelta", "dB", "dC", "dA", "checkpoints", "workspace", "z", "dz"):
        setattr(a, k, 4096)
    a.u_sb = a.delta_sb = a.dout_sb = a.z_sb = 32 * 64
    a.u_sl = a.delta_sl = a.dout_sl = a.z_sl = 64
    a.B_sb = a.C_sb = 32 * 16
    a.B_sl = a.C_sl = 16
    a.workspace_bytes = 1 << 40
    a.dz_sb, a.dz_sl = 32 * 128, 0                      # one stride without the other
    assert lib.swx_scan_bwd(a, None) == _lib.SWX_ERR_INVALID_ARG
    a.dz_sb, a.dz_sl = 32 * 128, 32                     # rows overlap
    assert lib.swx_scan_bwd(a, None) == _lib.SWX_ERR_INVALID_ARG
    c = _lib.ConvArgs()
    c.batch, c.seqlen, c.dim, c.width = 2, 32, 64, 4
    c.dtype = 0                                               # fp32
    for k in ("x", "weight", "dout", "dx", "dweight", "workspace"):
        setattr(c, k, 4096)
    c.x_sb, c.x_sl, c.dout_sb, c.dout_sl = 32 * 64, 64, 32 * 64, 64
    c.workspace_bytes = 1 << 40
    c.dx_sb, c.dx_sl = 0, 128
    assert lib.swx_conv1d_bwd(c, None) == _lib.SWX_ERR_INVALID_ARG


def test_header_is_plain_c_and_a_c_program_links_the_library(tmp_path):
    """A C caller (a cgo or JNI binding's shim) compiles include/swiftx_b200.h as strict
    C99, links the library, and sees the argument structs with the library's own sizes
    (host-only calls: no GPU needed)."""
    import shutil
    import subprocess
    if shutil.which("gcc") is None:
        pytest.skip("gcc not available")
    lib = _lib.load()
    src = tmp_path / "caller.c"
    src.write_text(
        '#include <stdio.h>\n#include "swiftx_b200.h"\n'
        "int main(void) {\n"
        "    printf(\"%d %lld %d %d %d %d\\n\", swx_abi_version(), (long long)swx_scan_checkpoint_floats(1, 17, 3),\n"
        "           swx_scan_fwd(NULL, NULL), (int)(swx_scan_args_size() == sizeof(swx_scan_args)),\n"
        "           (int)(swx_conv_args_size() == sizeof(swx_conv_args)),\n"
        "           (int)(swx_decode_args_size() == sizeof(swx_decode_args)));\n"
        "    return 0;\n}\n")
    libdir = os.path.dirname(lib._name)
    exe = tmp_path / "caller"
    subprocess.run(["gcc", "-std=c99", "-Wall", "-Wextra", "-pedantic", "-Werror", f"-I{ROOT}/include", str(src),
                    f"-L{libdir}", "-lswiftx_b200", f"-Wl,-rpath,{libdir}", "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split()
    assert out == ["13", "96", str(_lib.SWX_ERR_INVALID_ARG), "1", "1", "1"]
