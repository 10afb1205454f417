"""Layers shared by the library's models."""

from __future__ import annotations

import torch
import torch.nn.functional as F
from torch import nn


class TcLinear(nn.Linear):
    """``nn.Linear`` whose GEMMs run on the library's tcgen05 CTA-pair kernel.

    On bf16 CUDA inputs on sm_100 (bias-free), the forward ``x W^T`` and the input-gradient
    ``dy W`` are :func:`dattri_llm_b200.ops.linear.linear`; anything else is ``F.linear``.
    It is still an ``nn.Linear`` to the capture engine (``__bw_layer_type__``), and it
    declares ``__bw_fused_capture__``: while a LoGra capture watches it, the capture's
    projections are computed inside these GEMMs (see ``ops/linear.py``) instead of by
    separate launches that re-read the layer's input and output gradient.
    """

    __bw_layer_type__ = "nn.Linear"
    __bw_fused_capture__ = True

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        from dattri_llm_b200.ops import linear as tc

        if self.bias is not None or not tc.supported(x, self.weight):
            return F.linear(x, self.weight, self.bias)
        link = self.__dict__.get("_bw_capture_link") if tc.fused_capture_enabled() else None
        tail, slot = link.before_forward(self, x) if link is not None else (None, None)
        y, a_pt = tc.linear(x, self.weight, tail_t=tail, slot=slot)
        if link is not None:
            link.after_forward(self, a_pt, slot)
        return y


def tc_linearize(model: nn.Module) -> list[str]:
    """Turn every bias-free ``nn.Linear`` of *model* into a :class:`TcLinear` in place (the
    same parameters, hooks and names; only the GEMMs change).  Lets a Hugging Face model
    run its projections on the library's kernels.  Returns the converted module names."""
    done = []
    for name, module in model.named_modules():
        if type(module) is nn.Linear and module.bias is None:
            module.__class__ = TcLinear
            done.append(name)
    return done
