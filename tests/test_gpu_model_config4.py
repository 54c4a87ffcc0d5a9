"""benchmark config 4's layer shapes through the whole EquivariantTransformer, against the
reference model run on the CPU (tests/golden/model_config4.pt, made by make_golden.py).

In Repr([0,1],32), hidden Repr([0,1,2,3],128), 8 heads, 16-NN within each graph; 3 layers
(in -> hidden, hidden -> hidden, hidden -> out) on 4 graphs of 50 nodes.  Out Repr([0], 8):
the reference rejects 8 heads on the configured out mult 1 (attention.py:233-236).  The
weights are not stored: both sides fill every parameter from the same seeded recipe
(make_golden.seeded_parameters), which the identical parameter names make reproducible.
Tolerance: 1e-4 relative L2 (float32-level mix, bf16x3) and 2e-2 for the bf16-mix mode.
"""
from __future__ import annotations

import importlib.util
import os

import pytest
import torch

import flash_eq as fe
from conftest import GOLDEN, golden, rel_l2

pytestmark = pytest.mark.gpu


def _make_golden():
    spec = importlib.util.spec_from_file_location("make_golden", os.path.join(GOLDEN, "make_golden.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


@pytest.mark.parametrize("mix", ["bf16x3", "bf16"])
def test_config4_model_matches_reference(cuda_device, mix):
    fx = golden("model_config4.pt")
    dev = cuda_device
    model = fe.EquivariantTransformer(fe.Repr([0, 1], 32), fe.Repr([0, 1, 2, 3], 128), fe.Repr([0], 8),
                                      num_layers=fx["num_layers"], num_heads=fx["num_heads"], max_dist=10.0)
    _make_golden().seeded_parameters(model, fx["param_seed"])
    model = model.to(dev).eval()
    for m in model.modules():
        if isinstance(m, fe.EquivariantEdgewiseLinear):
            m.mix_precision = mix
    g = fe.Graph(src=fx["src"].to(dev), dst=fx["dst"].to(dev), num_nodes=fx["coords"].shape[0])
    caps = []
    h = model.layers[0].register_forward_hook(lambda m, i, o: caps.append(o))
    with torch.no_grad():
        y = model(fx["coords"].to(dev), fx["x"].to(dev), g)
    h.remove()
    tol = 1e-4 if mix == "bf16x3" else 2e-2
    assert rel_l2(caps[0], fx["first_layer_output"]) < tol
    assert rel_l2(y, fx["output"]) < tol
