"""Host-side logic of the LM harness (swiftx_b200.sift) that needs no GPU: the bf16
weight copies used under bf16 autocast (one buffer, one view per weight, refreshed in
place), the list of weights they cover, and when a block takes the fused mixer node."""
import torch

from swiftx_b200.sift import SiftConfig, SiftLM, _bf16_copies


def test_bf16_copies_map_each_weight_and_refresh_in_place():
    torch.manual_seed(0)
    ws = [torch.randn(5, 3), torch.randn(7), torch.randn(2, 2, 2)]
    views = _bf16_copies(ws)
    assert set(views) == {id(w) for w in ws}
    for w in ws:
        v = views[id(w)]
        assert v.dtype == torch.bfloat16 and v.shape == w.shape
        assert torch.equal(v, w.to(torch.bfloat16))
    flat = views[id(ws[0])]._base
    assert all(views[id(w)]._base is flat for w in ws)          # one buffer
    with torch.no_grad():
        ws[1].mul_(3.0)
    again = _bf16_copies(ws, flat=flat)                            # refresh in place
    assert again[id(ws[1])].data_ptr() == views[id(ws[1])].data_ptr()
    assert torch.equal(views[id(ws[1])], ws[1].to(torch.bfloat16))


def test_projection_weights_cover_every_bias_free_projection_and_the_head():
    m = SiftLM(SiftConfig(vocab_size=16, d_model=32, n_layers=2, d_state=8))
    ws = m.projection_weights()
    names = {id(p): n for n, p in m.named_parameters()}
    got = sorted(names[id(w)] for w in ws)
    want = sorted([f"backbone.layers.{i}.mixer.{k}.weight" for i in range(2)
                   for k in ("in_proj", "x_proj", "dt_proj", "out_proj")] + ["embedding.weight"])
    assert got == want                                            # the head is tied to the embedding
    m.half()
    assert m.projection_weights() is None                          # only fp32 weights get copies


def test_fused_mixer_node_only_where_its_kernels_apply(monkeypatch):
    """SiftBlock runs the mixer as one autograd node (_MixerCore) only when every one of
    its preconditions holds -- CUDA bf16 activations under autograd, bf16 copies of
    x_proj's and dt_proj's weights made, no SiftX pathway mix, no x_proj bias, a conv bias,
    an even d_inner (dz and the conv's dx land in the halves of one (b, L, 2 d_inner)
    buffer) -- and otherwise keeps the per-op graph.  The activations are stood in for
    by an object with the two attributes the check reads."""
    from types import SimpleNamespace

    from swiftx_b200 import sift
    from swiftx_b200.sift import SiftBlock

    cuda_bf16 = SimpleNamespace(is_cuda=True, dtype=torch.bfloat16)
    blk = SiftBlock(8, d_state=4)
    copies = {id(blk.x_proj.weight): torch.zeros(1), id(blk.dt_proj.weight): torch.ones(1)}
    monkeypatch.setattr(sift, "_W16", copies)
    w = blk._core_weights(cuda_bf16)
    assert w is not None and w[0] is copies[id(blk.x_proj.weight)] and w[1] is copies[id(blk.dt_proj.weight)]

    assert blk._core_weights(SimpleNamespace(is_cuda=False, dtype=torch.bfloat16)) is None
    assert blk._core_weights(SimpleNamespace(is_cuda=True, dtype=torch.float32)) is None
    with torch.no_grad():
        assert blk._core_weights(cuda_bf16) is None
    monkeypatch.setattr(sift, "_FUSED_CORE", False)
    assert blk._core_weights(cuda_bf16) is None
    monkeypatch.setattr(sift, "_FUSED_CORE", True)
    monkeypatch.setattr(sift, "_W16", None)
    assert blk._core_weights(cuda_bf16) is None
    monkeypatch.setattr(sift, "_W16", {id(blk.x_proj.weight): torch.zeros(1)})      # dt_proj's copy missing
    assert blk._core_weights(cuda_bf16) is None

    odd = SiftBlock(7, d_state=4, expand=1)                                          # d_inner 7
    no_conv_bias = SiftBlock(8, d_state=4, conv_bias=False)
    mixed = SiftBlock(8, d_state=4, timescales=[(1e-3, 1e-2), (1e-2, 1e-1)], pathway_gate=True)
    for other in (odd, no_conv_bias, mixed):
        monkeypatch.setattr(sift, "_W16", {id(other.x_proj.weight): torch.zeros(1),
                                           id(other.dt_proj.weight): torch.ones(1)})
        assert other._core_weights(cuda_bf16) is None
