"""The reference's behavioural test suite (tests/test_optimizer.py of the
reference project), re-stated for the CUDA drop-in: the same scenarios and
assertions, with models on cuda:0."""
import copy

import pytest
import torch
from torch import nn

from sandmuon_b200 import DiagonalWeightedPE, RankOneAWeightedPE, S8_COEFFICIENTS
from sandmuon_b200.optimizer import _s8_fp32

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


class _Proj(nn.Module):
    def __init__(self, rows, columns):
        super().__init__()
        self.proj = nn.Linear(columns, rows, bias=False)

    def forward(self, x):
        return self.proj(x)


def test_full_effective_batch_statistics_accumulate_over_microbatches():
    torch.manual_seed(10)
    model = _Proj(3, 4).to(DEV)
    x, target = torch.randn(9, 4, device=DEV), torch.randn(9, 3, device=DEV)
    prediction_before = model(x).detach()
    expected_b = (2 * (prediction_before - target) / x.shape[0]).square().mean(0)
    expected_b = expected_b / expected_b.mean()
    opt = RankOneAWeightedPE(model, lr=1e-3)
    opt.zero_grad(set_to_none=True)
    for start, end in ((0, 2), (2, 6), (6, 9)):
        ((model(x[start:end]) - target[start:end]).square().sum() / x.shape[0]).backward()
    before = model.proj.weight.detach().clone()
    opt.step()
    state = opt.state[model.proj.weight]
    torch.testing.assert_close(state["a_ema"], x.square().mean(0))
    torch.testing.assert_close(state["b_ema"], expected_b)
    assert state["a_count"] == state["b_count"] == 0
    assert not torch.equal(before, model.proj.weight)
    opt.close()


def _one_update(model, opt, x, target):
    opt.zero_grad(set_to_none=True)
    (model(x) - target).square().mean().backward()
    opt.step()


def test_optimizer_state_dict_resume_matches_continuous_updates():
    torch.manual_seed(11)
    model_a = nn.Sequential(nn.Linear(4, 5), nn.Tanh(), nn.Linear(5, 2)).to(DEV)
    opt_a = RankOneAWeightedPE(model_a, lr=2e-3)
    x, y = torch.randn(8, 4, device=DEV), torch.randn(8, 2, device=DEV)
    _one_update(model_a, opt_a, x, y)
    model_state = copy.deepcopy(model_a.state_dict())
    optimizer_state = copy.deepcopy(opt_a.state_dict())
    model_b = nn.Sequential(nn.Linear(4, 5), nn.Tanh(), nn.Linear(5, 2)).to(DEV)
    model_b.load_state_dict(model_state)
    opt_b = RankOneAWeightedPE(model_b, lr=2e-3)
    opt_b.load_state_dict(optimizer_state)
    _one_update(model_a, opt_a, x, y)
    _one_update(model_b, opt_b, x, y)
    for a, b in zip(model_a.parameters(), model_b.parameters()):
        torch.testing.assert_close(a, b)
    opt_a.close()
    opt_b.close()


@pytest.mark.parametrize("cls", [RankOneAWeightedPE, DiagonalWeightedPE])
def test_zero_signal_remains_finite(cls):
    model = _Proj(3, 4).to(DEV)
    opt = cls(model, lr=1e-3)
    opt.zero_grad(set_to_none=True)
    (model(torch.zeros(6, 4, device=DEV)) * 0).sum().backward()
    opt.step()
    for parameter in model.parameters():
        assert torch.isfinite(parameter).all()
    state = opt.state[model.proj.weight]
    keys = ("a_ema", "a_mean_ema", "b_ema") if cls is RankOneAWeightedPE else ("a_ema", "b_ema")
    for key in keys:
        assert torch.isfinite(state[key]).all()
    opt.close()


def test_s8_handles_both_orientations_and_zero_matrix():
    torch.manual_seed(13)
    for shape in ((7, 3), (3, 7), (4, 4)):
        x = torch.randn(2, *shape, device=DEV)
        y = _s8_fp32(x)
        assert y.shape == x.shape
        assert torch.isfinite(y).all()
    zero = _s8_fp32(torch.zeros(1, 4, 3, device=DEV))
    assert torch.equal(zero, torch.zeros_like(zero))


def test_qkv_share_activation_statistic_only_for_production_attention_names():
    class Attention(nn.Module):
        def __init__(self):
            super().__init__()
            self.q_proj = nn.Linear(4, 4, bias=False)
            self.k_proj = nn.Linear(4, 4, bias=False)
            self.v_proj = nn.Linear(4, 4, bias=False)

    class Block(nn.Module):
        def __init__(self):
            super().__init__()
            self.attn = Attention()
            self.cross_attn = Attention()

        def forward(self, x):
            return (self.attn.q_proj(x) + self.attn.k_proj(x) + self.attn.v_proj(x)
                    + self.cross_attn.q_proj(x) + self.cross_attn.k_proj(x) + self.cross_attn.v_proj(x))

    class Model(nn.Module):
        def __init__(self):
            super().__init__()
            self.transformer = nn.Module()
            self.transformer.h = nn.ModuleList([Block()])

        def forward(self, x):
            return self.transformer.h[0](x)

    torch.manual_seed(14)
    model = Model().to(DEV)
    block = model.transformer.h[0]
    opt = RankOneAWeightedPE(model, lr=1e-3)
    assert opt.a_sources[id(block.attn.k_proj.weight)] is block.attn.q_proj.weight
    assert opt.a_sources[id(block.attn.v_proj.weight)] is block.attn.q_proj.weight
    assert opt.a_sources[id(block.cross_attn.k_proj.weight)] is block.cross_attn.k_proj.weight
    x = torch.randn(5, 4, device=DEV)
    opt.zero_grad(set_to_none=True)
    model(x).square().mean().backward()
    opt.step()
    torch.testing.assert_close(opt.state[block.attn.q_proj.weight]["a_ema"], x.square().mean(0))
    assert "a_ema" not in opt.state[block.attn.k_proj.weight]
    opt.close()


@pytest.mark.parametrize("cls", [DiagonalWeightedPE, RankOneAWeightedPE])
@pytest.mark.parametrize("rows,columns", [(4, 4), (7, 3), (3, 7)])
def test_actual_update_norm_matches_frobenius_graft(cls, rows, columns):
    torch.manual_seed(15)
    lr = 1e-3
    model = _Proj(rows, columns).to(DEV)
    optimizer = cls(model, lr=lr)
    x, target = torch.randn(12, columns, device=DEV), torch.randn(12, rows, device=DEV)
    before = model.proj.weight.detach().clone()
    (model(x) - target).square().mean().backward()
    optimizer.step()
    update_norm = (model.proj.weight.detach() - before).norm() / lr
    torch.testing.assert_close(update_norm, torch.tensor(rows ** .5, device=DEV), rtol=2e-5, atol=2e-5)
    optimizer.close()


def test_step_closure_runs_with_grad_enabled_and_updates_parameters():
    torch.manual_seed(16)
    model = nn.Sequential(nn.Linear(4, 5), nn.Tanh(), nn.Linear(5, 2)).to(DEV)
    optimizer = RankOneAWeightedPE(model, lr=1e-3)
    x, target = torch.randn(7, 4, device=DEV), torch.randn(7, 2, device=DEV)
    before = [parameter.detach().clone() for parameter in model.parameters()]

    def closure():
        optimizer.zero_grad(set_to_none=True)
        loss = (model(x) - target).square().mean()
        loss.backward()
        return loss

    loss = optimizer.step(closure)
    assert torch.isfinite(loss)
    assert any(not torch.equal(old, new) for old, new in zip(before, model.parameters()))
    assert all(p.grad is not None and torch.isfinite(p.grad).all() for p in model.parameters())
    optimizer.close()


def test_state_keys_match_the_reference_layout():
    torch.manual_seed(17)
    model = nn.Sequential(nn.Linear(4, 5), nn.Tanh(), nn.Linear(5, 2)).to(DEV)
    for cls, a_keys in ((RankOneAWeightedPE, {"a_sum", "a_count", "a_first_sum", "a_ema", "a_mean_ema"}),
                        (DiagonalWeightedPE, {"a_sum", "a_count", "a_ema"})):
        opt = cls(model, lr=1e-3)
        _one_update(model, opt, torch.randn(6, 4, device=DEV), torch.randn(6, 2, device=DEV))
        w = model[0].weight
        assert set(opt.state[w]) == a_keys | {"b_sum", "b_count", "b_ema", "momentum_buffer"}
        assert set(opt.state[model[0].bias]) == {"exp_avg", "exp_avg_sq", "step"}
        assert isinstance(opt.state[model[0].bias]["step"], int)
        opt.close()


def test_coefficients_exported():
    assert len(S8_COEFFICIENTS) == 5 and all(len(abc) == 3 for abc in S8_COEFFICIENTS)
