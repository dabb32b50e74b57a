"""Parameters and gradients the kernels do not read directly: BF16 weights,
strided (transposed-view) weights and gradients.  The reference steps in FP32
on `gradient.float()` and adds `direction.to(parameter.dtype)` with alpha
-lr (sandmuon/optimizer.py:245-248, 281, 315); the B200 optimizer steps an
FP32 work copy and adds its update in the parameter's dtype, so

  * strided FP32 parameters and gradients give bitwise the same weights as
    contiguous ones;
  * a BF16 parameter ends at the reference's BF16 result, up to one BF16
    rounding step where the two round the update in a different order.
"""
import numpy as np
import pytest
import torch
from torch import nn

from sandmuon_b200 import RankOneAWeightedPE, _lib
from sandmuon_b200.workloads import synth_gpt_statistics

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")
LR = 1e-2


def _model(shapes, dtype=torch.float32, transposed=False):
    """nn.Sequential of bias-free Linear layers (out, in); with `transposed`
    every weight is a transposed view of an (in, out) tensor."""
    layers = []
    for d_out, d_in in shapes:
        lin = nn.Linear(d_in, d_out, bias=False)
        if transposed:
            lin.weight = nn.Parameter(torch.empty(d_in, d_out).t())
        layers.append(lin)
    model = nn.Sequential(*layers).to(DEV)
    return model.to(dtype)


def _fill(model, weights, grads, stats, opt, transposed_grads=False):
    with torch.no_grad():
        for i, lin in enumerate(model):
            lin.weight.copy_(torch.from_numpy(weights[i]))
            g = torch.from_numpy(grads[i]).to(DEV)
            if transposed_grads:
                g = g.t().contiguous().t()
            lin.weight.grad = g.to(lin.weight.dtype)
    from sandmuon_b200.workloads import inject_statistics
    inject_statistics(opt, stats)


SHAPES = [(256, 384), (640, 256), (384, 384)]


def _inputs():
    rng = np.random.default_rng(11)
    weights = [(rng.standard_normal(s) * 0.02).astype(np.float32) for s in SHAPES]
    grads = [(rng.standard_normal(s) * 1e-4).astype(np.float32) for s in SHAPES]
    return rng, weights, grads


def test_strided_parameters_and_gradients_match_contiguous_bitwise():
    _, weights, grads = _inputs()
    results = []
    for strided in (False, True):
        model = _model(SHAPES, transposed=strided)
        assert all(lin.weight.is_contiguous() != strided for lin in model)
        opt = RankOneAWeightedPE(model, lr=LR)
        stats = synth_gpt_statistics(opt, np.random.default_rng(5), count=4096, inject=False)
        for _ in range(2):
            _fill(model, weights, grads, stats, opt, transposed_grads=strided)
            opt.step()
        results.append([lin.weight.detach().contiguous().clone() for lin in model])
        assert all(opt.state[lin.weight]["momentum_buffer"].is_contiguous() for lin in model)
        opt.close()
    for a, b in zip(*results):
        assert torch.equal(a, b)
    assert _lib.device_status(DEV) == 0


def test_bf16_parameters_follow_reference_rounding():
    _, weights, grads = _inputs()
    weights = [torch.from_numpy(w).to(torch.bfloat16).float().numpy() for w in weights]   # representable in BF16
    grads = [torch.from_numpy(g).to(torch.bfloat16).float().numpy() for g in grads]
    stats = None
    runs = {}
    for dtype in (torch.float32, torch.bfloat16):
        model = _model(SHAPES, dtype=dtype)
        opt = RankOneAWeightedPE(model, lr=LR)
        if stats is None:
            stats = synth_gpt_statistics(opt, np.random.default_rng(5), count=4096, inject=False)
        _fill(model, weights, grads, stats, opt)
        before = [lin.weight.detach().float().clone() for lin in model]
        opt.step()
        runs[dtype] = (before, [lin.weight.detach().clone() for lin in model])
        opt.close()
    before32, after32 = runs[torch.float32]
    before16, after16 = runs[torch.bfloat16]
    for w0, w1, b0, b1 in zip(before32, after32, before16, after16):
        assert torch.equal(w0, b0)
        direction = (w0 - w1) / LR                      # the FP32 direction
        # the reference: param.add_(direction.to(bf16), alpha=-lr), in BF16
        want = b0.to(torch.bfloat16).add(direction.to(torch.bfloat16), alpha=-LR)
        got = b1
        assert got.dtype == torch.bfloat16
        diff = (got.float() - want.float()).abs()
        # The update is rounded to BF16 in a different order (before or after
        # the product with -lr, which is no power of two): the two updates
        # differ by up to one BF16 step of the update, and the final roundings
        # by one step of the result, so at most 2^-6 of the operands' scale.
        step = (b0.abs() + LR * direction.abs()) * 2.0 ** -6 + 1e-30
        worst = float((diff / step).max())
        equal = float((diff == 0).float().mean())
        assert worst <= 1.0 and equal > 0.95, (worst, equal)
    assert _lib.device_status(DEV) == 0
