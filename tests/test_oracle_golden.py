"""Pins the numpy oracle (oracle/sandmuon_oracle.py) to the reference's own
outputs, stored as golden fixtures by tests/golden/make_golden.py.  CPU only."""
from pathlib import Path

import numpy as np
import pytest

from oracle import sandmuon_oracle as orc

GOLDEN = Path(__file__).resolve().parent / "golden"


def load(name):
    return dict(np.load(GOLDEN / name))


def rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30)


def test_diagonal_inverse_sqrt_matches_reference():
    g = load("primitives.npz")
    for i in range(4):
        got = orc.diagonal_inverse_sqrt(g[f"dis_in_{i}"])
        np.testing.assert_allclose(got, g[f"dis_out_{i}"], rtol=2e-6, atol=0)
        assert np.isfinite(got).all()


def test_rank1_inverse_sqrt_matches_reference():
    g = load("primitives.npz")
    for i in range(2):
        inv, z, c = orc.rank1_inverse_sqrt(g[f"r1_second_{i}"], g[f"r1_mean_{i}"])
        np.testing.assert_allclose(inv, g[f"r1_inv_{i}"], rtol=2e-6)
        np.testing.assert_allclose(z, g[f"r1_z_{i}"], rtol=2e-6, atol=1e-7)
        np.testing.assert_allclose(c, g[f"r1_c_{i}"], rtol=2e-6)


def test_rank1_whiten_and_mapback_match_reference():
    g = load("primitives.npz")
    left = (g["wh_li"], g["wh_lz"], g["wh_lc"])
    right = (g["wh_ri"], g["wh_rz"], g["wh_rc"])
    np.testing.assert_allclose(orc.rank1_whiten(g["wh_src"], left, right), g["wh_out"], rtol=1e-5, atol=1e-6)
    left = (g["mb_li"], g["mb_lz"], g["mb_lc"])
    right = (g["mb_ri"], g["mb_rz"], g["mb_rc"])
    np.testing.assert_allclose(orc.rank1_mapback(g["mb_q"], left, right), g["mb_out"], rtol=1e-5, atol=1e-6)


def test_graft_matches_reference_and_norm_is_sqrt_rows():
    g = load("primitives.npz")
    got = orc.graft_direction(g["gr_in"], 7)
    np.testing.assert_allclose(got, g["gr_out"], rtol=2e-6)
    assert abs(np.linalg.norm(got) - np.sqrt(7)) < 1e-5


@pytest.mark.parametrize("case", range(8))
def test_s8_matches_reference(case):
    g = load("s8.npz")
    got = orc.s8_fp32(g[f"s8_in_{case}"])
    want = g[f"s8_out_{case}"]
    assert got.shape == want.shape
    assert rel(got, want) < 2e-5


def test_s8_zero_batch_gives_zeros():
    g = load("s8.npz")
    got = orc.s8_fp32(g["s8_zero_in"])
    assert np.array_equal(got, g["s8_zero_out"]) and not got.any()


def test_uneven_microbatch_statistics_and_step_match_reference():
    g = load("uneven_stats.npz")
    opt = orc.OracleSandMuon({"w": (40, 24)}, {"w": "w"}, rank_one_a=True, lr=1e-3)
    for m in range(3):
        opt.add_a("w", g[f"x/{m}"])
        opt.add_b("w", g[f"cot/{m}"])
    st = opt.state["w"]
    np.testing.assert_allclose(st["a_sum"], g["a_sum"], rtol=1e-5)
    np.testing.assert_allclose(st["a_first_sum"], g["a_first_sum"], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(st["b_sum"], g["b_sum"], rtol=1e-5)
    w = {"w": g["init"].copy()}
    opt.step(w, {"w": g["grad"]})
    for key in ("a_ema", "a_mean_ema", "b_ema", "momentum_buffer"):
        np.testing.assert_allclose(st[key], g[key], rtol=1e-5, atol=1e-7)
    assert st["a_count"] == st["b_count"] == 0
    assert rel(w["w"] - g["init"], g["w_after"] - g["init"]) < 1e-4


@pytest.mark.parametrize("variant", ["rank1", "diag"])
def test_mini_gpt_three_steps_match_reference(variant):
    """Replays the reference's recorded gradients and statistics-producing
    rows through the oracle and compares weights and state after each step."""
    import torch
    from mini_models import MiniGPT, gpt_matrix_names

    g = load(f"mini_gpt_{variant}.npz")
    layers = 2
    names = gpt_matrix_names(layers)
    model = MiniGPT(layers)
    shapes = {n: tuple(p.shape) for n, p in model.named_parameters()}
    a_source = {}
    for n in names:
        a_source[n] = n.replace("k_proj", "q_proj").replace("v_proj", "q_proj") if ".attn." in n else n
    aux = [n for n in shapes if n not in names]
    opt = orc.OracleSandMuon({n: shapes[n] for n in names}, a_source, aux, rank_one_a=(variant == "rank1"),
                             lr=float(g["lr"]))
    weights = {n: g[f"init/{n}"].copy() for n in shapes}
    # per-module inputs/cotangents are reproduced with a CPU forward of the
    # same model in float32 (the reference's hooks saw exactly these rows)
    with torch.no_grad():
        for n, p in model.named_parameters():
            p.copy_(torch.from_numpy(weights[n]))
    for s in range(int(g["steps"])):
        rows_in, rows_out = {}, {}
        hooks = []
        for mname, module in model.named_modules():
            if isinstance(module, torch.nn.Linear):
                def fwd(mod, inp, out, mname=mname):
                    rows_in.setdefault(mname, []).append(inp[0].detach().reshape(-1, inp[0].shape[-1]).numpy().copy())
                    out.register_hook(lambda grad, mname=mname: rows_out.setdefault(mname, []).append(
                        grad.detach().reshape(-1, grad.shape[-1]).numpy().copy()))
                hooks.append(module.register_forward_hook(fwd))
        model.zero_grad(set_to_none=True)
        for m in range(int(g["micro"])):
            x = torch.from_numpy(g[f"x/{s}/{m}"])
            cot = torch.from_numpy(g[f"cot/{s}/{m}"])
            (model(x) * cot).sum().div(int(g["micro"])).backward()
        for h in hooks:
            h.remove()
        for n in names:
            mod = n[: -len(".weight")]
            if a_source[n] == n:
                for r in rows_in[mod]:
                    opt.add_a(n, r)
            for r in rows_out[mod]:
                opt.add_b(n, r)
        grads = {n: g[f"grad/{s}/{n}"] for n in shapes}
        opt.step(weights, grads)
        for n in shapes:
            ref_w = g[f"w/{s}/{n}"]
            assert rel(weights[n], ref_w) < 1e-4, (s, n, rel(weights[n], ref_w))
        for n in names:
            st = opt.state[n]
            for key in ("b_ema", "momentum_buffer"):
                np.testing.assert_allclose(st[key], g[f"state/{s}/{n}/{key}"], rtol=1e-4, atol=1e-6)
            if a_source[n] == n:
                np.testing.assert_allclose(st["a_ema"], g[f"state/{s}/{n}/a_ema"], rtol=1e-4, atol=1e-7)
        with torch.no_grad():
            for n, p in model.named_parameters():
                p.copy_(torch.from_numpy(weights[n]))


def test_oracle_follows_reference_gpt2_training_run():
    """The oracle as the optimizer of the small config-2 GPT-2 model (FP32 torch
    forward/backward on CPU, hooks feeding add_a / add_b): every step's loss
    and the recorded matrices after the last step match the reference
    optimizer's own run (tests/golden/gpt2_small.npz)."""
    import re

    import torch

    from sandmuon_b200.workloads import GPT2, gpt2_matrix_filter
    g = load("gpt2_small.npz")
    steps, lr = int(g["steps"]), float(g["lr"])
    torch.manual_seed(0)
    model = GPT2(layers=2, width=128, heads=4, vocab=512, context=64)
    params = dict(model.named_parameters())
    with torch.no_grad():
        for n, p in params.items():
            p.copy_(torch.from_numpy(g[f"init/{n}"]))
    modules = {n + ".weight": m for n, m in model.named_modules() if gpt2_matrix_filter(n, m)}
    sharing = re.compile(r"^(transformer\.h\.\d+\.attn\.)[kv]_proj\.weight$")
    source = {}
    for n in modules:
        m = sharing.match(n)
        source[n] = m.group(1) + "q_proj.weight" if m else n
    aux = [n for n in params if n not in modules]
    oracle = orc.OracleSandMuon({n: tuple(params[n].shape) for n in modules}, source, aux, rank_one_a=True, lr=lr)
    captured_a, captured_b = {}, {}

    def hook(name):
        def fwd(module, inputs, output):
            if source[name] == name:
                captured_a.setdefault(name, []).append(inputs[0].detach().reshape(-1, inputs[0].shape[-1]).numpy())
            output.register_hook(lambda grad: captured_b.setdefault(name, []).append(
                grad.detach().reshape(-1, grad.shape[-1]).numpy()))
        return fwd

    handles = [m.register_forward_hook(hook(n)) for n, m in modules.items()]
    batches = [torch.from_numpy(g[f"tokens/{i}"]) for i in range(2)]
    threads = torch.get_num_threads()
    torch.set_num_threads(1)  # the fixture was recorded single-threaded
    try:
        for s in range(steps):
            captured_a.clear()
            captured_b.clear()
            model.zero_grad(set_to_none=True)
            total = 0.0
            for b in batches:
                logits = model(b[:, :-1])
                loss = torch.nn.functional.cross_entropy(logits.reshape(-1, 512), b[:, 1:].reshape(-1)) / 2
                loss.backward()
                total += float(loss.detach())
            assert abs(total - float(g[f"loss/{s}"])) / float(g[f"loss/{s}"]) < 1e-4, (s, total)
            for n, rows in captured_a.items():
                for r in rows:
                    oracle.add_a(n, r)
            for n, rows in captured_b.items():
                for r in rows:
                    oracle.add_b(n, r)
            weights = {n: p.detach().numpy().copy() for n, p in params.items()}
            grads = {n: p.grad.detach().numpy() for n, p in params.items() if p.grad is not None}
            oracle.step(weights, grads)
            with torch.no_grad():
                for n, p in params.items():
                    p.copy_(torch.from_numpy(weights[n]))
    finally:
        torch.set_num_threads(threads)
        for h in handles:
            h.remove()
    for key in g:
        if key.startswith("final/"):
            n = key[len("final/"):]
            assert rel(params[n].detach().numpy() - g[f"init/{n}"], g[key] - g[f"init/{n}"]) < 1e-3, n
