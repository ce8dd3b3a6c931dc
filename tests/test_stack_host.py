"""The hybrid stack harness on the host: its state dict has the reference's names and shapes
(recorded in the stack fixtures from the reference's own model), so a reference checkpoint loads
unchanged.  Nothing here launches a kernel."""
from __future__ import annotations

from pathlib import Path

import numpy as np
import torch

from visionstack_b200 import Qwen3_5TextConfig
from visionstack_b200 import workloads as W
from visionstack_b200.stack import Qwen3_5TextModel

GOLDEN = Path(__file__).resolve().parent / "golden"


def test_stack_state_dict_matches_reference():
    ref = np.load(GOLDEN / "stack_tiny_f32.npz")
    with torch.device("meta"):
        model = Qwen3_5TextModel(Qwen3_5TextConfig(**W.STACK_TINY))
    ours = {k: str(tuple(v.shape)) for k, v in model.state_dict().items()}
    theirs = dict(zip(ref["names"].tolist(), ref["shapes"].tolist()))
    assert ours == theirs


def test_stack_layer_types_and_full_size_shapes():
    cfg = Qwen3_5TextConfig(**W.STACK_48)
    assert cfg.layer_types.count("full_attention") == 12 and cfg.layer_types.count("linear_attention") == 36
    with torch.device("meta"):
        model = Qwen3_5TextModel(cfg)
    n = sum(p.numel() for p in model.parameters())
    assert 5.0e9 < n < 5.6e9
    assert tuple(model.layers[3].self_attn.q_proj.weight.shape) == (16 * 256 * 2, 2048)
    assert tuple(model.layers[0].linear_attn.in_proj_qkv.weight.shape) == (8192, 2048)


def test_stack_params_do_not_depend_on_order():
    shapes = {"b.weight": (3, 4), "a.weight": (2, 2), "x.A_log": (4,)}
    p1 = W.make_stack_params(shapes, 7, "f32")
    p2 = W.make_stack_params(dict(reversed(list(shapes.items()))), 7, "f32")
    for k in shapes:
        assert np.array_equal(p1[k], p2[k])
