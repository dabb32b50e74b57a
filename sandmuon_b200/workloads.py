"""Synthetic workloads of the benchmark configurations (seeded numpy).

Used by bench.py and the tests to build the config-1 / config-4 matrix sets
and the accumulated hook statistics they would have after a number of
microbatches.  Statistics are drawn like config 0: per-channel activation mean
~ N(0.1, 0.05^2) and std ~ LogNormal(0, 0.5); per-output-channel cotangent
scale 1e-3 * LogNormal(0, 0.5).  Not used by the optimizer itself.
"""
from __future__ import annotations

import numpy as np
import torch
from torch import nn


def gpt_matrix_model(layers: int, width: int, hidden: int) -> nn.Module:
    """Module tree with the historical GPT names (q/k/v/o, mlp.c_fc, mlp.c_proj)
    holding only the bias-free Linear weights the optimizer selects."""
    root = nn.Module()
    root.transformer = nn.Module()
    blocks = []
    for _ in range(layers):
        blk = nn.Module()
        blk.attn = nn.Module()
        for proj in ("q_proj", "k_proj", "v_proj", "o_proj"):
            setattr(blk.attn, proj, nn.Linear(width, width, bias=False))
        blk.mlp = nn.Module()
        blk.mlp.c_fc = nn.Linear(width, hidden, bias=False)
        blk.mlp.c_proj = nn.Linear(hidden, width, bias=False)
        blocks.append(blk)
    root.transformer.h = nn.ModuleList(blocks)
    return root


CONFIGS = {
    "cfg1": dict(layers=9, width=768, hidden=3072, microbatches=8, rows=16 * 1024),
    "cfg4": dict(layers=24, width=2048, hidden=8192, microbatches=8, rows=8 * 2048),
}


def synth_gpt_statistics(opt, rng: np.random.Generator, count: int, *, inject: bool = True) -> dict:
    """Accumulated sums of `count` rows for every matrix of `opt`; when
    `inject`, also writes them into opt.state like the hooks would.

    Returns {name: dict(a_sum, a_first_sum, a_count, b_sum, b_count)} with the
    a_* entries only for activation-statistic sources."""
    out = {}
    for name, p in opt.named_matrices.items():
        d_out, d_in = p.shape
        entry = {}
        source = opt.a_sources[id(p)]
        if source is p:
            mean = rng.normal(0.1, 0.05, d_in)
            std = np.exp(rng.normal(0.0, 0.5, d_in))
            noise = 1.0 + 0.01 * rng.standard_normal(d_in)
            entry["a_sum"] = (count * (mean ** 2 + std ** 2) * noise).astype(np.float32)
            entry["a_first_sum"] = (count * mean * noise).astype(np.float32)
            entry["a_count"] = count
        scale = 1e-3 * np.exp(rng.normal(0.0, 0.5, d_out))
        entry["b_sum"] = (count * scale ** 2 * (1.0 + 0.01 * rng.standard_normal(d_out))).astype(np.float32)
        entry["b_count"] = count
        out[name] = entry
    if inject:
        inject_statistics(opt, out)
    return out


def inject_statistics(opt, stats: dict) -> None:
    """Writes accumulated sums into opt.state (the hooks' state layout)."""
    for name, entry in stats.items():
        p = opt.named_matrices[name]
        st = opt.state[p]
        if "a_sum" in entry:
            for key in ("a_sum", "a_first_sum"):
                if key == "a_first_sum" and not opt.rank_one_a:
                    continue
                t = torch.from_numpy(entry[key]).to(p.device)
                if key in st and st[key].shape == t.shape:
                    st[key].copy_(t, non_blocking=True)
                else:
                    st[key] = t
            st["a_count"] = int(entry["a_count"])
        t = torch.from_numpy(entry["b_sum"]).to(p.device)
        if "b_sum" in st and st["b_sum"].shape == t.shape:
            st["b_sum"].copy_(t, non_blocking=True)
        else:
            st["b_sum"] = t
        st["b_count"] = int(entry["b_count"])


def s8_dense_flops(shapes) -> float:
    """Dense tensor-core FLOPs of the engine's S8 precision schedule per
    matrix, summed: 13 x (4 r^2 c + 2 r^3) with r <= c -- stages 1-4 run
    their three products (X X^T, G G, P X) compensated (three BF16 products
    each), stage 5 plain.  Symmetric products are counted dense; the engine
    computes only their upper block triangle (sm_s8_executed_flops gives the
    executed count).  Used as the relative cost of a matrix when sharding."""
    total = 0.0
    for rows, cols in shapes:
        r, c = min(rows, cols), max(rows, cols)
        total += 13.0 * (4.0 * r * r * c + 2.0 * r ** 3)
    return total


# ------------------------------------------------------------ config 2: GPT-2

class CausalSelfAttention(nn.Module):
    """Bias-free q/k/v/o projections around torch's fused causal attention."""

    def __init__(self, width: int, heads: int):
        super().__init__()
        self.heads = heads
        for proj in ("q_proj", "k_proj", "v_proj", "o_proj"):
            setattr(self, proj, nn.Linear(width, width, bias=False))

    def forward(self, x):
        b, t, c = x.shape
        q, k, v = (p(x).view(b, t, self.heads, c // self.heads).transpose(1, 2)
                   for p in (self.q_proj, self.k_proj, self.v_proj))
        y = torch.nn.functional.scaled_dot_product_attention(q, k, v, is_causal=True)
        return self.o_proj(y.transpose(1, 2).reshape(b, t, c))


class GPT2Block(nn.Module):
    def __init__(self, width: int, heads: int, hidden: int):
        super().__init__()
        self.ln_1 = nn.LayerNorm(width)
        self.attn = CausalSelfAttention(width, heads)
        self.ln_2 = nn.LayerNorm(width)
        self.mlp = nn.Module()
        self.mlp.c_fc = nn.Linear(width, hidden, bias=False)
        self.mlp.c_proj = nn.Linear(hidden, width, bias=False)

    def forward(self, x):
        x = x + self.attn(self.ln_1(x))
        return x + self.mlp.c_proj(torch.nn.functional.gelu(self.mlp.c_fc(self.ln_2(x))))


class GPT2(nn.Module):
    """GPT-2-style decoder of benchmark configuration 2 (historical parameter names, so
    q/k/v statistic sharing applies): token and position embeddings, pre-LN
    blocks of bias-free Linear layers, final LayerNorm, and an output head
    tied to the token embedding.  Random initialisation (N(0, 0.02^2)); the
    SandMuon matrices are the transformer.h.* Linear weights, everything else
    (embeddings, LayerNorms) trains with the AdamW auxiliaries."""

    def __init__(self, layers: int = 9, width: int = 768, heads: int = 12, vocab: int = 50257,
                 context: int = 1024):
        super().__init__()
        self.transformer = nn.Module()
        self.transformer.wte = nn.Embedding(vocab, width)
        self.transformer.wpe = nn.Embedding(context, width)
        self.transformer.h = nn.ModuleList([GPT2Block(width, heads, 4 * width) for _ in range(layers)])
        self.transformer.ln_f = nn.LayerNorm(width)
        for name, p in self.named_parameters():
            if p.ndim == 2:
                nn.init.normal_(p, std=0.02)

    def forward(self, idx):
        t = idx.shape[1]
        pos = torch.arange(t, device=idx.device)
        x = self.transformer.wte(idx) + self.transformer.wpe(pos)
        for block in self.transformer.h:
            x = block(x)
        return self.transformer.ln_f(x) @ self.transformer.wte.weight.t()


def gpt2_matrix_filter(name: str, module: nn.Module) -> bool:
    """module_filter of the config-2 run: the Linear layers of the blocks."""
    return name.startswith("transformer.h.") and isinstance(module, nn.Linear)


def gpt2_train_step(model: nn.Module, opt, batches, targets) -> torch.Tensor:
    """One optimizer step over microbatches (BF16 autocast forward/backward,
    FP32 weights): mean cross-entropy over the microbatches, backward per
    microbatch (the hooks accumulate statistics), opt.step(), zero_grad.
    Returns the step's summed loss as a device tensor."""
    total = torch.zeros((), device=batches[0].device)
    n = len(batches)
    for idx, tgt in zip(batches, targets):
        with torch.autocast("cuda", dtype=torch.bfloat16):
            logits = model(idx)
            loss = torch.nn.functional.cross_entropy(logits.view(-1, logits.shape[-1]), tgt.view(-1)) / n
        loss.backward()
        total += loss.detach()
    opt.step()
    opt.zero_grad(set_to_none=True)
    return total
