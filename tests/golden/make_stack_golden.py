"""Generate ``stack_tiny_f32.npz`` / ``stack_tiny_bf16.npz`` by running the reference's text
stack (ShadowBoxer/models/qwen35/text.py, ``Qwen3_5TextModel``) on the host.

    python tests/golden/make_stack_golden.py --ref <reference checkout>

The 4-layer stack of ``visionstack_b200.workloads.STACK_TINY`` (three Gated DeltaNet layers and
one gated attention layer) gets the seeded parameters of ``make_stack_params`` and runs the calls
of ``make_stack_calls``: a 70-token prefill into a hybrid cache, three decode steps, one 4-token
step, and a cache-less 40-token call under a 2-D mask.  Stored: every call's
``last_hidden_state``, the final DeltaNet states of layer 0 and the key cache of layer 3, plus the
state-dict names and shapes (the drop-in check).
"""
from __future__ import annotations

import argparse
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO))

from visionstack_b200 import workloads as W  # noqa: E402


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("VISIONSTACK_REF"),
                    help="checkout of the reference (or set VISIONSTACK_REF)")
    args = ap.parse_args()
    if not args.ref:
        ap.error("give --ref <reference checkout> or set VISIONSTACK_REF")
    sys.path.insert(0, os.path.join(args.ref, "ShadowBoxer"))
    import torch

    torch.set_num_threads(max(1, os.cpu_count() or 1))
    from models.qwen35.cache import Qwen3_5HybridCache
    from models.qwen35.config import Qwen3_5TextConfig
    from models.qwen35.text import Qwen3_5TextModel

    tdt = {"f32": torch.float32, "bf16": torch.bfloat16}
    for dtype in ("f32", "bf16"):
        torch.manual_seed(0)
        cfg = Qwen3_5TextConfig(**W.STACK_TINY)
        model = Qwen3_5TextModel(cfg).eval().to(tdt[dtype])
        shapes = {k: tuple(v.shape) for k, v in model.state_dict().items()}
        params = W.make_stack_params(shapes, seed=7, dtype=dtype)
        sd = {k: torch.from_numpy(v) if k.endswith(("A_log", "dt_bias")) else torch.from_numpy(v).to(tdt[dtype])
              for k, v in params.items()}
        model.load_state_dict(sd, strict=True)
        for k in ("A_log", "dt_bias"):  # kept float32, as the reference loader does
            for mod in model.modules():
                if hasattr(mod, k):
                    getattr(mod, k).data = getattr(mod, k).data.float()
        ids, spans, mask = W.make_stack_calls(W.STACK_TINY)
        out = {"names": np.array(sorted(shapes)), "shapes": np.array([str(shapes[k]) for k in sorted(shapes)])}
        with torch.inference_mode():
            cache = Qwen3_5HybridCache()
            for i, (a, b) in enumerate(spans):
                o = model(input_ids=torch.from_numpy(ids[:, a:b]), past_key_values=cache, use_cache=True)
                out[f"h{i}"] = o.last_hidden_state.float().numpy()
            out["rec0"] = cache.recurrent_states[0].float().numpy()
            out["conv0"] = cache.conv_states[0].float().numpy()
            out["key3"] = cache.key_cache[3].float().numpy()
            o = model(input_ids=torch.from_numpy(ids[:, :40]), attention_mask=torch.from_numpy(mask))
            out["h_mask"] = o.last_hidden_state.float().numpy()
        out["torch_version"] = np.array(torch.__version__)
        np.savez_compressed(HERE / f"stack_tiny_{dtype}.npz", **out)
        print(dtype, {k: (v.shape, float(np.abs(v).max()), bool(np.isfinite(v).all()))
                      for k, v in out.items() if k.startswith(("h", "rec", "key", "conv"))})
        print("param dtypes", sorted({str(p.dtype) for p in model.parameters()}))


if __name__ == "__main__":
    main()
