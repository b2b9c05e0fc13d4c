"""Host-side logic of the LM harness (swiftx_b200.sift) that needs no GPU: the bf16
weight copies used under bf16 autocast (one buffer, one view per weight, refreshed in
place) and the list of weights they cover."""
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
