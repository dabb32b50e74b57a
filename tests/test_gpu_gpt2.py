"""The drop-in optimizer inside a real training loop (benchmark configuration
2 at a small size): a GPT-2-style decoder with fused causal attention, BF16 autocast
forward/backward over several microbatches, tied embeddings and LayerNorms on
the AdamW auxiliaries.  Checks that the hooks' statistics equal torch
reductions of the tensors they saw (1e-5 relative), that q/k/v share one
activation statistic, that a step consumes and zeroes every sum, and that an
FP32 training run follows the reference's own recorded run of the same model
(tests/golden/gpt2_small.npz)."""
from pathlib import Path

import numpy as np
import pytest
import torch

from sandmuon_b200 import RankOneAWeightedPE
from sandmuon_b200.workloads import GPT2, gpt2_matrix_filter

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")
GOLDEN = Path(__file__).resolve().parent / "golden"
STAT_REL = 1e-5


def rel(a, b):
    a, b = a.double(), b.double()
    return float((a - b).norm() / b.norm().clamp_min(1e-300))


def small_gpt2():
    torch.manual_seed(3)
    return GPT2(layers=2, width=128, heads=4, vocab=512, context=64).to(DEV)


def test_hook_statistics_match_torch_under_autocast():
    model = small_gpt2()
    opt = RankOneAWeightedPE(model, lr=1e-2, module_filter=gpt2_matrix_filter)
    seen_in, seen_out = {}, {}
    probes = []
    for name, module in model.named_modules():
        if gpt2_matrix_filter(name, module):
            def fwd(mod, inp, out, key=name + ".weight"):
                seen_in.setdefault(key, []).append(inp[0].detach().reshape(-1, inp[0].shape[-1]).float().clone())
                out.register_hook(lambda g, key=key: seen_out.setdefault(key, []).append(
                    g.detach().reshape(-1, g.shape[-1]).float().clone()))
            probes.append(module.register_forward_hook(fwd))
    gen = torch.Generator(device=DEV).manual_seed(4)
    for _ in range(3):
        idx = torch.randint(0, 512, (4, 64), generator=gen, device=DEV)
        tgt = torch.randint(0, 512, (4, 64), generator=gen, device=DEV)
        with torch.autocast("cuda", dtype=torch.bfloat16):
            logits = model(idx)
            loss = torch.nn.functional.cross_entropy(logits.view(-1, 512), tgt.view(-1)) / 3
        loss.backward()
    for h in probes:
        h.remove()
    torch.cuda.synchronize()
    params = dict(model.named_parameters())
    for name, p in opt.named_matrices.items():
        st = opt.state[p]
        src = opt.a_sources[id(p)]
        if src is p:
            x = torch.cat(seen_in[name])
            assert st["a_count"] == x.shape[0]
            assert rel(st["a_sum"], x.square().sum(0)) < STAT_REL, name
            assert rel(st["a_first_sum"], x.sum(0)) < STAT_REL, name
        else:
            assert "a_sum" not in st and name.split(".attn.")[1][0] in "kv"
            assert src is params[name.replace("k_proj", "q_proj").replace("v_proj", "q_proj")]
        d = torch.cat(seen_out[name])
        assert st["b_count"] == d.shape[0]
        assert rel(st["b_sum"], d.square().sum(0)) < STAT_REL, name
    opt.step()
    torch.cuda.synchronize()
    for p in opt.named_matrices.values():
        st = opt.state[p]
        assert float(st["b_sum"].abs().sum()) == 0.0 and st["b_count"] == 0
        if "a_sum" in st:
            assert float(st["a_sum"].abs().sum()) == 0.0 and st["a_count"] == 0
    opt.close()


def test_training_trajectory_matches_reference_golden_run():
    """FP32 forward/backward (TF32 off) from the reference run's initial
    weights and tokens: every step's loss within 1e-2 relative of the
    reference's, and the accumulated update of the recorded matrices within
    3e-2 relative Frobenius error, cosine >= 0.999."""
    g = dict(np.load(GOLDEN / "gpt2_small.npz"))
    steps, lr = int(g["steps"]), float(g["lr"])
    model = small_gpt2()
    params = dict(model.named_parameters())
    with torch.no_grad():
        for n, p in params.items():
            p.copy_(torch.from_numpy(g[f"init/{n}"]))
    batches = [torch.from_numpy(g[f"tokens/{i}"]).to(DEV) for i in range(2)]
    opt = RankOneAWeightedPE(model, lr=lr, module_filter=gpt2_matrix_filter)
    tf32 = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        for s in range(steps):
            total = 0.0
            for b in batches:
                logits = model(b[:, :-1])
                loss = torch.nn.functional.cross_entropy(logits.reshape(-1, 512), b[:, 1:].reshape(-1)) / 2
                loss.backward()
                total += float(loss)
            opt.step()
            opt.zero_grad(set_to_none=True)
            ref = float(g[f"loss/{s}"])
            assert abs(total - ref) / ref < 1e-2, (s, total, ref)
    finally:
        torch.backends.cuda.matmul.allow_tf32 = tf32
    for key in g:
        if key.startswith("final/"):
            n = key[len("final/"):]
            d = (params[n].detach().cpu() - torch.from_numpy(g[f"init/{n}"])).double().flatten()
            d_ref = torch.from_numpy(g[key] - g[f"init/{n}"]).double().flatten()
            assert rel(d, d_ref) < 3e-2, (n, rel(d, d_ref))
            assert float(d @ d_ref / (d.norm() * d_ref.norm())) > 0.999, n
    opt.close()
