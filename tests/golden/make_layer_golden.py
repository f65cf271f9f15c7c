"""Generate ``tests/golden/layer_*.npz`` from the REFERENCE's torch GLA layer.

    TOPS_REF=/path/to/pallas-kernel python tests/golden/make_layer_golden.py

The reference layer's JAX code cannot run here (no JAX); its torch gold
``tests/src/layers/gla.py:53`` (the layer its tests compare against) is imported from
the read-only reference tree, given the seeded weights of ``layer_cases.py``, and run in
fp32: the fixture stores the output, the input gradient of loss = sum(o * do) and the
parameter gradients (only the small ones for ``small_grads`` cases).  Nothing at test
time needs the reference.
"""
from __future__ import annotations

import os
import sys

import numpy as np

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
import layer_cases as LC  # noqa: E402

REF = os.environ.get("TOPS_REF", "/root/reference")


def main():
    import torch
    sys.path.insert(0, REF)
    from tests.src.layers.gla import GatedLinearAttention  # type: ignore
    here = os.path.dirname(os.path.abspath(__file__))
    for name, case in LC.LAYER_CASES.items():
        torch.manual_seed(0)
        layer = GatedLinearAttention(mode="chunk", **case["args"], layer_idx=0)
        shapes = [(n, tuple(p.shape)) for n, p in layer.named_parameters()]
        W = LC.weights(shapes, case["seed"])
        with torch.no_grad():
            for n, p in layer.named_parameters():
                p.copy_(torch.from_numpy(W[n]))
        x, do, mask = LC.inputs(case)
        xt = torch.from_numpy(x).requires_grad_()
        mt = None if mask is None else torch.from_numpy(mask)
        o, _, _ = layer(xt, attention_mask=mt)
        (o * torch.from_numpy(do)).sum().backward()
        out = {"o": o.detach().numpy(), "dx": xt.grad.numpy()}
        for n, p in layer.named_parameters():
            if not case.get("small_grads") or p.numel() <= 8192:
                out["grad." + n] = p.grad.numpy()
        np.savez_compressed(os.path.join(here, name + ".npz"), **out)
        print(name, {k: v.shape for k, v in out.items()})


if __name__ == "__main__":
    main()
