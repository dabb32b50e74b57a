"""Small models shared by tests/golden/make_golden.py and the parity tests.

MiniGPT uses the historical GPT parameter names
(transformer.h.<i>.attn.{q,k,v,o}_proj, transformer.h.<i>.mlp.c_{fc,proj})
so the q/k/v activation-statistic sharing rule fires, plus LayerNorm
parameters that become AdamW auxiliaries.  It is a toy mixer, not attention:
only the parameter layout matters to the optimizer.
"""
from __future__ import annotations

import torch
from torch import nn


class Attention(nn.Module):
    def __init__(self, d):
        super().__init__()
        self.q_proj = nn.Linear(d, d, bias=False)
        self.k_proj = nn.Linear(d, d, bias=False)
        self.v_proj = nn.Linear(d, d, bias=False)
        self.o_proj = nn.Linear(d, d, bias=False)

    def forward(self, x):
        q, k, v = self.q_proj(x), self.k_proj(x), self.v_proj(x)
        return self.o_proj(torch.tanh(q) * k + v)


class MLP(nn.Module):
    def __init__(self, d, hidden):
        super().__init__()
        self.c_fc = nn.Linear(d, hidden, bias=False)
        self.c_proj = nn.Linear(hidden, d, bias=False)

    def forward(self, x):
        return self.c_proj(torch.nn.functional.gelu(self.c_fc(x)))


class Block(nn.Module):
    def __init__(self, d, hidden):
        super().__init__()
        self.attn = Attention(d)
        self.mlp = MLP(d, hidden)

    def forward(self, x):
        x = x + self.attn(x)
        return x + self.mlp(x)


class MiniGPT(nn.Module):
    def __init__(self, layers=2, d=32, hidden=128):
        super().__init__()
        self.transformer = nn.Module()
        self.transformer.h = nn.ModuleList([Block(d, hidden) for _ in range(layers)])
        self.transformer.ln_f = nn.LayerNorm(d)

    def forward(self, x):
        for block in self.transformer.h:
            x = block(x)
        return self.transformer.ln_f(x)


def gpt_matrix_names(layers: int) -> list[str]:
    names = []
    for i in range(layers):
        for proj in ("q_proj", "k_proj", "v_proj", "o_proj"):
            names.append(f"transformer.h.{i}.attn.{proj}.weight")
        names += [f"transformer.h.{i}.mlp.c_fc.weight", f"transformer.h.{i}.mlp.c_proj.weight"]
    return names
