"""The reference's ChainRules rrules (src/chainrules.jl:31-123, src/grad_generate_vals.jl:291-305)
as torch.autograd Functions over the B200 path, so any torch loss composes with them.

    logdet_of_vals(prob, vals)                 -> generate_logdet with vals replaced
    inv_quadratic_loss_of_vals(prob, vals, y)  -> 0.5*||generate_inv(y)||^2 with vals replaced
    generate_of_vals(prob, vals, xi)           -> generate with vals replaced (d/dvals and d/dxi)
    generate_t(prob, xi)                       -> generate with the d/dxi pullback
"""
from __future__ import annotations

import torch

from . import api
from .problem import GraphGPProblem, set_vals


def _with_vals(prob: GraphGPProblem, vals: torch.Tensor) -> GraphGPProblem:
    return set_vals(prob, vals.detach().to(prob.device, prob.torch_dtype).contiguous())


class _LogdetOfVals(torch.autograd.Function):
    @staticmethod
    def forward(ctx, vals, prob):
        p2 = _with_vals(prob, vals)
        ld, g = api.generate_logdet_and_grad_vals(p2)
        ctx.save_for_backward(g if isinstance(g, torch.Tensor) else torch.as_tensor(g))
        return torch.tensor(ld, dtype=vals.dtype, device=vals.device)

    @staticmethod
    def backward(ctx, gy):
        (g,) = ctx.saved_tensors
        return g.to(gy.device, gy.dtype) * gy, None


class _InvQuadLossOfVals(torch.autograd.Function):
    @staticmethod
    def forward(ctx, vals, prob, data):
        p2 = _with_vals(prob, vals)
        loss, g = api.generate_inv_loss_grad_vals(p2, data)
        ctx.save_for_backward(g if isinstance(g, torch.Tensor) else torch.as_tensor(g))
        return torch.tensor(loss, dtype=vals.dtype, device=vals.device)

    @staticmethod
    def backward(ctx, gy):
        (g,) = ctx.saved_tensors
        return g.to(gy.device, gy.dtype) * gy, None, None


class _GenerateOfVals(torch.autograd.Function):
    @staticmethod
    def forward(ctx, vals, xi, prob):
        p2 = _with_vals(prob, vals)
        ctx.prob = p2
        ctx.save_for_backward(xi)
        return api.generate(p2, xi.detach())

    @staticmethod
    def backward(ctx, gy):
        (xi,) = ctx.saved_tensors
        gy = gy.contiguous()
        dvals = api.generate_grad_vals(ctx.prob, xi.detach(), gy) \
            if ctx.needs_input_grad[0] else None
        dxi = api.generate_grad_xi(ctx.prob, gy) if ctx.needs_input_grad[1] else None
        return dvals, dxi, None


class _Generate(torch.autograd.Function):
    @staticmethod
    def forward(ctx, xi, prob):
        ctx.prob = prob
        return api.generate(prob, xi.detach())

    @staticmethod
    def backward(ctx, gy):
        return api.generate_grad_xi(ctx.prob, gy.contiguous()), None


def logdet_of_vals(prob: GraphGPProblem, vals: torch.Tensor) -> torch.Tensor:
    return _LogdetOfVals.apply(vals, prob)


def inv_quadratic_loss_of_vals(prob: GraphGPProblem, vals: torch.Tensor, data) -> torch.Tensor:
    return _InvQuadLossOfVals.apply(vals, prob, data)


def generate_of_vals(prob: GraphGPProblem, vals: torch.Tensor, xi: torch.Tensor) -> torch.Tensor:
    return _GenerateOfVals.apply(vals, xi, prob)


def generate_t(prob: GraphGPProblem, xi: torch.Tensor) -> torch.Tensor:
    return _Generate.apply(xi, prob)
