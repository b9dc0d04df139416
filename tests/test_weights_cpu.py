"""Raw GPT-2 weight loading (Gpt2Layer.load_weights / load_stack): file
naming, [in, out] -> [out, in] transposition, size checks, partial files.
The last test loads the reference's own `layer_weights/` biases where the
reference tree is checked out beside this repository (skipped elsewhere)."""
import os
import sys

import numpy as np
import pytest

torch = pytest.importorskip("torch")

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
from oracle.oracle import reference_root  # noqa: E402

REF_WEIGHTS = os.path.join(reference_root(), "layer_weights")


def test_load_weights_transposes_and_reports(gae, tmp_path):
    D, H, F = 256, 4, 1024
    layer = gae.Gpt2Layer.random(D, H, F, device="cpu", seed=1)
    rng = np.random.default_rng(0)
    w_fc = rng.standard_normal((D, F)).astype(np.float32)  # GPT-2 layout [in, out]
    b_fc = rng.standard_normal(F).astype(np.float32)
    b_proj = rng.standard_normal(D).astype(np.float32)
    w_fc.tofile(tmp_path / "w_fc_layer3.bin")
    b_fc.tofile(tmp_path / "b_fc_layer3.bin")
    b_proj.tofile(tmp_path / "b_proj_layer3.bin")
    before = layer.w["w_qkv"].clone()
    loaded = layer.load_weights(str(tmp_path), 3)
    assert sorted(loaded) == ["b_fc", "b_fc2", "w_fc"]
    assert torch.equal(layer.w["w_fc"], torch.from_numpy(w_fc).t().to(torch.bfloat16))
    assert torch.equal(layer.w["b_fc"], torch.from_numpy(b_fc))
    assert torch.equal(layer.w["b_fc2"], torch.from_numpy(b_proj))
    assert torch.equal(layer.w["w_qkv"], before)  # absent files leave tensors alone
    assert layer.load_weights(str(tmp_path), 4) == []


def test_load_weights_rejects_wrong_size(gae, tmp_path):
    layer = gae.Gpt2Layer.random(256, 4, 1024, device="cpu")
    np.zeros(1000, np.float32).tofile(tmp_path / "b_fc_layer0.bin")
    with pytest.raises(gae.GAEError):
        layer.load_weights(str(tmp_path), 0)


@pytest.mark.skipif(not os.path.isdir(REF_WEIGHTS), reason="reference tree not checked out here")
def test_reference_layer_weights_load():
    import __graft_entry__ as ge
    gae = ge.load_package()
    layers, report = gae.Gpt2Layer.load_stack(REF_WEIGHTS, 12, 768, 12, 3072, device="cpu")
    assert all(sorted(r) == ["b_fc", "b_fc2"] for r in report.values())
    for l in layers:
        assert torch.isfinite(l.w["b_fc"]).all() and float(l.w["b_fc"].abs().max()) > 0
    # layers differ from one another (each file is its own layer's)
    assert not torch.equal(layers[0].w["b_fc"], layers[1].w["b_fc"])
