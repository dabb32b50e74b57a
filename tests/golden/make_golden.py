"""Generates the golden fixtures in tests/golden/ by running the REFERENCE.

Run where a checkout of the SandMuon project exists, naming its root:

    SANDMUON_REFERENCE=<checkout> python tests/golden/make_golden.py [fixture ...]

It imports the reference package under the module name `sandmuon_ref` (to
avoid clashing with any other `sandmuon`), evaluates its public helpers and
optimizers on seeded inputs, and writes compressed .npz files next to this
script.  The GPU test machines never run this script; tests only read the
fixtures.
"""
from __future__ import annotations

import importlib.util
import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
from mini_models import MiniGPT  # noqa: E402


def load_reference():
    checkout = os.environ.get("SANDMUON_REFERENCE")
    if not checkout:
        raise SystemExit("set SANDMUON_REFERENCE to the root of a SandMuon checkout")
    root = Path(checkout) / "sandmuon"
    spec = importlib.util.spec_from_file_location("sandmuon_ref", root / "__init__.py",
                                                  submodule_search_locations=[str(root)])
    module = importlib.util.module_from_spec(spec)
    sys.modules["sandmuon_ref"] = module
    spec.loader.exec_module(module)
    import sandmuon_ref.optimizer as ref_opt  # noqa: E402
    return module, ref_opt


def np32(t):
    return t.detach().to(torch.float32).cpu().numpy().copy()


def primitives(ref):
    g = torch.Generator().manual_seed(101)
    out = {}
    vecs = [torch.rand(7, generator=g) + .3, torch.zeros(4), torch.logspace(-6, 3, 11),
            torch.rand(33, generator=g) * torch.rand(33, generator=g)]
    for i, v in enumerate(vecs):
        out[f"dis_in_{i}"] = np32(v)
        out[f"dis_out_{i}"] = np32(ref.diagonal_inverse_sqrt(v))
    for i, n in enumerate((6, 17)):
        x = torch.randn(500, n, generator=g) + torch.randn(n, generator=g)
        second, mean = x.square().mean(0), x.mean(0)
        inv, z, c = ref.rank1_inverse_sqrt(second, mean)
        out.update({f"r1_second_{i}": np32(second), f"r1_mean_{i}": np32(mean), f"r1_inv_{i}": np32(inv),
                    f"r1_z_{i}": np32(z), f"r1_c_{i}": np32(c)})
    src = torch.randn(2, 6, 4, generator=g)
    left = ref.rank1_inverse_sqrt(torch.rand(6, generator=g) + .3, torch.randn(6, generator=g) * .2)
    right = ref.rank1_inverse_sqrt(torch.rand(4, generator=g) + .3, torch.randn(4, generator=g) * .2)
    out["wh_src"] = np32(src)
    for k, (a, b) in enumerate(zip(("li", "lz", "lc"), ("ri", "rz", "rc"))):
        out[f"wh_{a}"] = np32(left[k])
        out[f"wh_{b}"] = np32(right[k])
    out["wh_out"] = np32(ref.rank1_whiten(src, left, right))
    q = torch.randn(5, 3, generator=g)
    l5 = ref.rank1_inverse_sqrt(torch.rand(5, generator=g) + .3, torch.randn(5, generator=g) * .1)
    r3 = ref.rank1_inverse_sqrt(torch.rand(3, generator=g) + .3, torch.randn(3, generator=g) * .1)
    out["mb_q"] = np32(q)
    for k, (a, b) in enumerate(zip(("li", "lz", "lc"), ("ri", "rz", "rc"))):
        out[f"mb_{a}"] = np32(l5[k])
        out[f"mb_{b}"] = np32(r3[k])
    out["mb_out"] = np32(ref.rank1_mapback(q, l5, r3))
    val = torch.randn(7, 3, generator=g)
    out["gr_in"] = np32(val)
    out["gr_out"] = np32(ref._graft_direction(val, 7))
    return out


def s8_cases(ref):
    g = torch.Generator().manual_seed(202)
    out = {}
    shapes = [(2, 7, 3), (2, 3, 7), (2, 4, 4), (3, 16, 48), (3, 48, 16), (2, 64, 64), (2, 96, 160), (1, 130, 70)]
    for i, shape in enumerate(shapes):
        x = torch.randn(*shape, generator=g)
        # anisotropic columns and a rank-one spike, like the benchmark's S8 sweep
        x = x * torch.exp(torch.randn(shape[-1], generator=g))
        u = torch.randn(shape[0], shape[1], 1, generator=g)
        v = torch.randn(shape[0], 1, shape[2], generator=g)
        x = x + 3.0 * u * v
        out[f"s8_in_{i}"] = np32(x)
        out[f"s8_out_{i}"] = np32(ref._s8_fp32(x))
    out["s8_zero_in"] = np.zeros((1, 4, 3), np.float32)
    out["s8_zero_out"] = np32(ref._s8_fp32(torch.zeros(1, 4, 3)))
    return out


def mini_gpt_run(ref_pkg, *, rank_one, layers=2, d=32, hidden=128, steps=3, micro=3, rows=24, seed=303, lr=1e-2):
    torch.manual_seed(seed)
    model = MiniGPT(layers, d, hidden)
    g = torch.Generator().manual_seed(seed + 1)
    cls = ref_pkg.RankOneAWeightedPE if rank_one else ref_pkg.DiagonalWeightedPE
    opt = cls(model, lr=lr)
    out = {"lr": np.float32(lr), "steps": np.int64(steps), "micro": np.int64(micro)}
    for name, p in model.named_parameters():
        out[f"init/{name}"] = np32(p)
    for s in range(steps):
        opt.zero_grad(set_to_none=True)
        for m in range(micro):
            x = torch.randn(rows + m, d, generator=g) * (1 + torch.rand(d, generator=g)) + 0.1
            cot = torch.randn(rows + m, d, generator=g)
            out[f"x/{s}/{m}"] = np32(x)
            out[f"cot/{s}/{m}"] = np32(cot)
            (model(x) * cot).sum().div(micro).backward()
        for name, p in model.named_parameters():
            out[f"grad/{s}/{name}"] = np32(p.grad)
        opt.step()
        for name, p in model.named_parameters():
            out[f"w/{s}/{name}"] = np32(p)
        names = {id(p): n for n, p in model.named_parameters()}
        for p, st in opt.state.items():
            for key, val in st.items():
                if isinstance(val, torch.Tensor):
                    out[f"state/{s}/{names[id(p)]}/{key}"] = np32(val)
    opt.close()
    return out


def uneven_stats(ref_pkg):
    """Microbatches of 2, 4, 3 rows through Linear(24 -> 40) (the reference's
    accumulation test shape, scaled up), recording sums before the step."""
    torch.manual_seed(404)
    model = torch.nn.Sequential(torch.nn.Linear(24, 40, bias=False))
    opt = ref_pkg.RankOneAWeightedPE(model, lr=1e-3)
    g = torch.Generator().manual_seed(405)
    out = {"init": np32(model[0].weight)}
    opt.zero_grad(set_to_none=True)
    for m, n in enumerate((2, 4, 3)):
        x = torch.randn(n, 24, generator=g) + 0.5
        cot = torch.randn(n, 40, generator=g)
        out[f"x/{m}"], out[f"cot/{m}"] = np32(x), np32(cot)
        (model(x) * cot).sum().backward()
    st = opt.state[model[0].weight]
    out["a_sum"], out["a_first_sum"], out["b_sum"] = np32(st["a_sum"]), np32(st["a_first_sum"]), np32(st["b_sum"])
    out["grad"] = np32(model[0].weight.grad)
    opt.step()
    out["w_after"] = np32(model[0].weight)
    for key in ("a_ema", "a_mean_ema", "b_ema", "momentum_buffer"):
        out[key] = np32(st[key])
    opt.close()
    return out


def gpt2_run(ref_pkg, *, steps=6, seed=3, lr=2e-2):
    """The reference RankOneAWeightedPE training a small GPT-2-style decoder
    (2 layers, width 128, 4 heads, vocab 512; the config-2 model family of
    sandmuon_b200.workloads.GPT2) in FP32 on two fixed batches of next-token
    prediction: initial weights, tokens, the summed loss of every step, and
    two SandMuon matrices after the last step."""
    sys.path.insert(0, str(HERE.parents[1]))
    from sandmuon_b200.workloads import GPT2, gpt2_matrix_filter
    torch.manual_seed(seed)
    model = GPT2(layers=2, width=128, heads=4, vocab=512, context=64)
    opt = ref_pkg.RankOneAWeightedPE(model, lr=lr, module_filter=gpt2_matrix_filter)
    g = torch.Generator().manual_seed(seed + 2)
    batches = [torch.randint(0, 512, (4, 64), generator=g) for _ in range(2)]
    out = {"lr": np.float32(lr), "steps": np.int64(steps)}
    for name, p in model.named_parameters():
        out[f"init/{name}"] = np32(p)
    for i, b in enumerate(batches):
        out[f"tokens/{i}"] = b.numpy().astype(np.int64)
    for s in range(steps):
        total = 0.0
        for b in batches:
            logits = model(b[:, :-1])
            loss = torch.nn.functional.cross_entropy(logits.reshape(-1, 512), b[:, 1:].reshape(-1)) / len(batches)
            loss.backward()
            total += float(loss.detach())
        opt.step()
        opt.zero_grad(set_to_none=True)
        out[f"loss/{s}"] = np.float64(total)
    for name in ("transformer.h.0.attn.q_proj.weight", "transformer.h.1.mlp.c_fc.weight"):
        out[f"final/{name}"] = np32(dict(model.named_parameters())[name])
    opt.close()
    return out


def main():
    """python tests/golden/make_golden.py [fixture ...]  (default: all)."""
    ref_pkg, ref_opt = load_reference()
    torch.set_num_threads(1)
    fixtures = {
        "primitives": lambda: primitives(ref_opt),
        "s8": lambda: s8_cases(ref_opt),
        "mini_gpt_rank1": lambda: mini_gpt_run(ref_pkg, rank_one=True),
        "mini_gpt_diag": lambda: mini_gpt_run(ref_pkg, rank_one=False),
        "uneven_stats": lambda: uneven_stats(ref_pkg),
        "gpt2_small": lambda: gpt2_run(ref_pkg),
    }
    for name in sys.argv[1:] or list(fixtures):
        np.savez_compressed(HERE / f"{name}.npz", **fixtures[name]())
    for f in sorted(HERE.glob("*.npz")):
        print(f.name, f.stat().st_size)


if __name__ == "__main__":
    main()
