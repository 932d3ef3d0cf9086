"""``nn.Linear`` drop-in whose product runs through ozaki2_int8_matmul
(the reference's fp_emulation/nn.py:7-47, same names and behaviour)."""
import torch
from torch import nn

from fp_emulation.ozaki import ozaki2_int8_matmul


class Linear(nn.Linear):
    """nn.Linear with float64 parameters whose x @ W^T is emulated on INT8 tensor
    cores.  Keeps nn.Linear's parameter names, so state_dicts are interchangeable."""

    def __init__(self, in_features, out_features, bias=True, device=None):
        super().__init__(in_features, out_features, bias=bias, device=device, dtype=torch.float64)

    def forward(self, x):
        x = x.to(torch.float64)
        lead = x.shape[:-1]
        # W^T is a transposed view: its columns are W's rows, contiguous along K,
        # which the split kernel reads directly (no copy).
        y = ozaki2_int8_matmul(x.reshape(-1, x.shape[-1]), self.weight.T)
        y = y.reshape(*lead, self.out_features)
        if self.bias is not None:
            y = y + self.bias
        return y


def convert(model):
    """Replace every nn.Linear inside ``model`` (recursively, in place) by
    :class:`Linear`, copying weights and bias as float64 and keeping their
    ``requires_grad``.  Returns ``model``."""
    for name, child in model.named_children():
        if isinstance(child, nn.Linear) and not isinstance(child, Linear):
            swapped = Linear(child.in_features, child.out_features, bias=child.bias is not None,
                             device=child.weight.device)
            swapped.weight.data.copy_(child.weight.data.to(torch.float64))
            swapped.weight.requires_grad_(child.weight.requires_grad)
            if child.bias is not None:
                swapped.bias.data.copy_(child.bias.data.to(torch.float64))
                swapped.bias.requires_grad_(child.bias.requires_grad)
            setattr(model, name, swapped)
        else:
            convert(child)
    return model
