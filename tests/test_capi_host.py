"""CPU tests of the boundary: the C-ABI library builds, loads and exports every
symbol include/sandmuon_b200.h declares; host-side logic of the optimizer
(selection, sharing, errors raised before device work); constants agree."""
import ctypes
import re
from pathlib import Path

import pytest
import torch
from torch import nn

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "sandmuon_b200.h"


def declared_symbols():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^[A-Za-z_][\w\s\*]*?\b(sm_\w+)\s*\(", text, flags=re.M)))


def test_header_declares_the_documented_entry_points():
    names = declared_symbols()
    for required in ("sm_version", "sm_last_error", "sm_stats_accumulate", "sm_plan_create", "sm_plan_step",
                     "sm_plan_destroy", "sm_s8_polar", "sm_adamw_multi", "sm_gemm_bf16"):
        assert required in names


def test_library_loads_and_exports_every_declared_symbol(built_library):
    lib = ctypes.CDLL(str(built_library))
    missing = [n for n in declared_symbols() if not hasattr(lib, n)]
    assert not missing, missing
    lib.sm_version.restype = ctypes.c_int
    assert lib.sm_version() == 3


def test_binding_signatures_cover_the_header(built_library):
    from sandmuon_b200 import _lib
    assert set(_lib.SIGNATURES) == set(declared_symbols())
    lib = _lib.load()
    assert lib.sm_version() == 3


STRUCTS = ("SmMatrixSpec", "SmStatSpec", "SmPlanSpec", "SmStepArgs", "SmCopySpec", "SmDeltaSpec", "SmAdamTensor")


def test_ctypes_structs_match_c_layout(tmp_path):
    """Every POD struct of the header: the ctypes binding has the size and the
    field offsets gcc computes for the C declaration."""
    import json
    import shutil
    import subprocess
    from sandmuon_b200 import _lib
    gcc = shutil.which("gcc") or shutil.which("cc")
    if gcc is None:
        pytest.skip("no C compiler")
    lines = ["#include <stdio.h>", "#include <stddef.h>", '#include "sandmuon_b200.h"', "int main(void) {",
             '  printf("{");']
    for i, name in enumerate(STRUCTS):
        fields = [f for f, _ in getattr(_lib, name)._fields_]
        offs = ", ".join(f'\\"{f}\\": %zu' for f in fields)
        args = ", ".join(f"offsetof({name}, {f})" for f in fields)
        sep = "," if i else ""
        lines.append(f'  printf("{sep}\\"{name}\\": {{\\"size\\": %zu, {offs}}}", sizeof({name}), {args});')
    lines += ['  printf("}\\n");', "  return 0;", "}"]
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines) + "\n")
    exe = tmp_path / "layout"
    subprocess.run([gcc, "-I", str(HEADER.parent), str(src), "-o", str(exe)], check=True)
    c_layout = json.loads(subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout)
    for name in STRUCTS:
        cls = getattr(_lib, name)
        assert c_layout[name]["size"] == ctypes.sizeof(cls), name
        for field, _ in cls._fields_:
            assert c_layout[name][field] == getattr(cls, field).offset, (name, field)


def test_engine_constants_match_package_constants():
    from sandmuon_b200 import S8_COEFFICIENTS, S8_MARGIN
    src = (ROOT / "sandmuon_b200" / "csrc" / "libsandmuon_b200.cu").read_text()
    block = src[src.index("kS8Coeff[5][3]"):]
    block = block[:block.index("};")]
    numbers = [float(x) for x in re.findall(r"-?\d+\.\d+", block)]
    assert numbers == [v for abc in S8_COEFFICIENTS for v in abc]
    assert f"kS8Margin = {S8_MARGIN}f" in src


class _Tiny(nn.Module):
    def __init__(self):
        super().__init__()
        self.proj = nn.Linear(4, 3, bias=False)
        self.norm = nn.LayerNorm(3)

    def forward(self, x):
        return self.norm(self.proj(x))


def test_selection_groups_and_defaults_match_reference():
    from sandmuon_b200 import DiagonalWeightedPE, RankOneAWeightedPE
    model = _Tiny()
    opt = RankOneAWeightedPE(model, lr=1e-3)
    assert opt.rank_one_a and opt.statistic_beta == .97
    assert opt.param_groups[0]["params"] == [model.proj.weight]
    assert opt.param_groups[0]["momentum"] == .8 and opt.param_groups[0]["use_muon"]
    assert opt.param_groups[1]["use_muon"] is False and opt.param_groups[1]["weight_decay"] == .01
    assert opt.param_groups[1]["adamw_lr_ratio"] == .1 and opt.param_groups[1]["adamw_betas"] == (.9, .999)
    opt.close()
    opt = DiagonalWeightedPE(model, lr=1e-3, module_filter=lambda n, m: n == "proj")
    assert not opt.rank_one_a
    opt.close()


def test_no_eligible_weights_raises_value_error():
    from sandmuon_b200 import RankOneAWeightedPE
    with pytest.raises(ValueError, match="No eligible trainable linear weights found"):
        RankOneAWeightedPE(nn.Sequential(nn.LayerNorm(3)), lr=1e-3)


def test_qkv_sharing_only_for_production_attention_names():
    from mini_models import MiniGPT
    from sandmuon_b200 import RankOneAWeightedPE
    model = MiniGPT(2, 8, 16)
    opt = RankOneAWeightedPE(model, lr=1e-3)
    for i in range(2):
        attn = model.transformer.h[i].attn
        assert opt.a_sources[id(attn.k_proj.weight)] is attn.q_proj.weight
        assert opt.a_sources[id(attn.v_proj.weight)] is attn.q_proj.weight
        assert opt.a_sources[id(attn.o_proj.weight)] is attn.o_proj.weight
    opt.close()


def test_step_errors_are_raised_before_device_work():
    """Missing / mismatched statistics raise the reference's RuntimeErrors from
    host-side counters alone (CPU model, so any device call would also fail)."""
    from sandmuon_b200 import RankOneAWeightedPE
    model = nn.Sequential(nn.Linear(4, 3, bias=False))
    opt = RankOneAWeightedPE(model, lr=1e-3)
    model[0].weight.grad = torch.zeros(3, 4)
    with pytest.raises(RuntimeError, match="Missing activation statistics: 0.weight"):
        opt.step()
    opt.state[model[0].weight].update(a_count=5, b_count=4)
    with pytest.raises(RuntimeError, match="Missing or mismatched cotangent statistics: 0.weight; expected 5, got 4"):
        opt.step()
    opt.close()


def test_cpu_tensors_fail_loudly_instead_of_falling_back():
    from sandmuon_b200 import RankOneAWeightedPE
    model = nn.Sequential(nn.Linear(4, 3, bias=False))
    opt = RankOneAWeightedPE(model, lr=1e-3)
    with pytest.raises(RuntimeError, match="CUDA"):
        model(torch.randn(2, 4)).sum().backward()
    opt.close()


def test_functional_helpers_keep_reference_semantics_on_cpu():
    from oracle import sandmuon_oracle as orc
    from sandmuon_b200.optimizer import (_graft_direction, diagonal_inverse_sqrt, rank1_inverse_sqrt,
                                         rank1_mapback, rank1_whiten)
    g = torch.Generator().manual_seed(3)
    v = torch.rand(9, generator=g) + .1
    torch.testing.assert_close(diagonal_inverse_sqrt(v), torch.from_numpy(orc.diagonal_inverse_sqrt(v.numpy())))
    s, m = torch.rand(6, generator=g) + .5, torch.randn(6, generator=g) * .2
    for a, b in zip(rank1_inverse_sqrt(s, m), orc.rank1_inverse_sqrt(s.numpy(), m.numpy())):
        torch.testing.assert_close(a, torch.as_tensor(b), rtol=1e-5, atol=1e-7)
    left, right = rank1_inverse_sqrt(s, m), rank1_inverse_sqrt(s[:4] + .1, m[:4])
    src = torch.randn(2, 6, 4, generator=g)
    want = orc.rank1_whiten(src.numpy(), [t.numpy() for t in left], [t.numpy() for t in right])
    torch.testing.assert_close(rank1_whiten(src, left, right), torch.from_numpy(want), rtol=1e-5, atol=1e-6)
    want = orc.rank1_mapback(src[0].numpy(), [t.numpy() for t in left], [t.numpy() for t in right])
    torch.testing.assert_close(rank1_mapback(src[0], left, right), torch.from_numpy(want), rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(_graft_direction(src[0], 6).norm(), torch.tensor(6 ** .5))
