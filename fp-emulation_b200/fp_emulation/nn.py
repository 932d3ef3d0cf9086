"""``nn.Linear`` drop-in whose product runs through ozaki2_int8_matmul
(the reference's fp_emulation/nn.py:7-47, same names and behaviour)."""
import torch
from torch import nn

from fp_emulation.ozaki import PreparedOperand, _ozaki2_forward, _ozaki2_forward_prepared, ozaki2_int8_matmul


class Linear(nn.Linear):
    """nn.Linear with float64 parameters whose x @ W^T is emulated on INT8 tensor
    cores.  Keeps nn.Linear's parameter names, so state_dicts are interchangeable.

    When autograd is not recording (``torch.no_grad()``, or nothing requires a
    gradient) the bias add is fused into the product's epilogue; the result is
    bit-identical to the reference's ``ozaki2_int8_matmul(x, W.T) + bias``.
    ``cache_weight_residues=True`` additionally keeps the split (int8 residues
    and column exponents) of the weight between such calls -- n_mod bytes per
    weight element -- and re-splits only when the weight's storage or version
    changes (an optimizer step, ``load_state_dict``, any in-place update)."""

    def __init__(self, in_features, out_features, bias=True, device=None, cache_weight_residues=False):
        super().__init__(in_features, out_features, bias=bias, device=device, dtype=torch.float64)
        self.cache_weight_residues = cache_weight_residues
        self._weight_op = None  # (the weight Parameter it was made for, PreparedOperand of W^T)

    def _records_grad(self, x):
        return torch.is_grad_enabled() and (
            x.requires_grad or self.weight.requires_grad or (self.bias is not None and self.bias.requires_grad))

    def _weight_operand(self):
        """W^T as a prepared right operand: W [out, in] row-major is B^T of the
        product, so B's columns are W's rows (K contiguous)."""
        if self._weight_op is None or self._weight_op[0] is not self.weight:
            self._weight_op = (self.weight, PreparedOperand(self.weight.detach().T, "right"))
        return self._weight_op[1]

    def forward(self, x):
        x = x.to(torch.float64)
        lead = x.shape[:-1]
        x2d = x.reshape(-1, x.shape[-1])
        if self._records_grad(x2d):
            # W^T is a transposed view: its columns are W's rows, contiguous along K,
            # which the split kernel reads directly (no copy).
            y = ozaki2_int8_matmul(x2d, self.weight.T)
            if self.bias is not None:
                y = y + self.bias
        elif self.cache_weight_residues and self.in_features > 0:
            y = _ozaki2_forward_prepared(x2d, self._weight_operand(), bias=self.bias)
        else:
            y = _ozaki2_forward(x2d, self.weight.T, bias=self.bias)
        return y.reshape(*lead, self.out_features)


def convert(model, cache_weight_residues=False):
    """Replace every nn.Linear inside ``model`` (recursively, in place) by
    :class:`Linear`, copying weights and bias as float64 and keeping their
    ``requires_grad``.  Returns ``model``.  ``cache_weight_residues`` is passed
    to every new layer (off by default, as in the reference, which has no such
    cache)."""
    for name, child in model.named_children():
        if isinstance(child, nn.Linear) and not isinstance(child, Linear):
            swapped = Linear(child.in_features, child.out_features, bias=child.bias is not None,
                             device=child.weight.device, cache_weight_residues=cache_weight_residues)
            swapped.weight.data.copy_(child.weight.data.to(torch.float64))
            swapped.weight.requires_grad_(child.weight.requires_grad)
            if child.bias is not None:
                swapped.bias.data.copy_(child.bias.data.to(torch.float64))
                swapped.bias.requires_grad_(child.bias.requires_grad)
            setattr(model, name, swapped)
        else:
            convert(child, cache_weight_residues)
    return model
