"""The reference's scripts import flow_expert / triton_gemm / cudagraph /
quant by bare name; dropin.install() maps those names to this package."""
import ast
import copy
import os
import sys

import pytest
import torch

from embodied_efficiency_b200 import dropin

# [file, module, name] of every aliased import in the reference's kernel/*.py
# (made by tests/golden/make_reference_imports.py from the reference checkout)
REF_IMPORTS = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "reference_imports.json")


@pytest.fixture
def installed():
    saved = {k: sys.modules.get(k) for k in dropin.ALIASES}
    mods = dropin.install()
    yield mods
    for k, v in saved.items():
        if v is None:
            sys.modules.pop(k, None)
        else:
            sys.modules[k] = v


def test_aliases_expose_expected_names(installed):
    for alias, names in dropin.EXPECTED.items():
        mod = installed[alias]
        for n in names:
            assert hasattr(mod, n), (alias, n)


def test_every_name_the_reference_imports_exists(installed):
    """Every `from <alias> import <name>` of the reference's kernel/*.py
    resolves in the aliased module."""
    import json
    triples = json.load(open(REF_IMPORTS))
    assert len(triples) > 10
    missing = [(fn, mod, name) for fn, mod, name in triples if not hasattr(installed[mod], name)]
    assert not missing, missing


def test_quantlinear_buffers_and_model_swap():
    from embodied_efficiency_b200.expert import ActionExpert, ActionExpertConfig
    from embodied_efficiency_b200.quant import QuantLinear, quantize_model, quantize_weight
    torch.manual_seed(0)
    lin = torch.nn.Linear(256, 64)
    ql = QuantLinear(lin, 4)
    q, s, gs = quantize_weight(lin.weight.data.float(), 4)
    assert torch.equal(ql.q, q) and torch.equal(ql.scale, s) and ql.gs == gs == 128
    assert ql.weight_bytes() == q.numel() * 0.5 + s.numel() * 2
    assert set(dict(ql.named_buffers())) == {"q", "scale"}
    m = quantize_model(ActionExpert(ActionExpertConfig(d_model=256, n_layers=1, n_heads=4, prefix_len=8)), 8)
    assert isinstance(m.in_proj, torch.nn.Linear) and isinstance(m.out_proj, torch.nn.Linear)
    assert isinstance(m.blocks[0].qkv, QuantLinear)
    copy.deepcopy(m)  # the reference's compiler deep-copies experts


@pytest.mark.gpu
def test_reference_compiler_flow_on_this_package(cuda, installed):
    """The calls kernel/compiler.py:search makes (seeded expert, deepcopy +
    quantize_model_triton, flow_sample, GraphedSampler) through the aliases;
    the reference's QuantLinear (quant.quantize_model) path agrees with the
    fused-kernel path."""
    import cudagraph
    import flow_expert
    import quant
    import triton_gemm
    cfg = flow_expert.ActionExpertConfig()
    cfg.d_model = 256
    torch.manual_seed(0)
    base = flow_expert.ActionExpert(cfg).to(cuda).to(torch.bfloat16).eval()
    x = torch.randn(1, cfg.horizon, cfg.action_dim, device=cuda, dtype=torch.bfloat16)
    ref = flow_expert.flow_sample(base, x, 10, base.encode_prefix(1)).float()
    m4 = triton_gemm.quantize_model_triton(copy.deepcopy(base), bits=4)
    q4 = quant.quantize_model(copy.deepcopy(base), 4)
    a = flow_expert.flow_sample(m4, x, 10, m4.encode_prefix(1)).float()
    b = flow_expert.flow_sample(q4, x, 10, q4.encode_prefix(1)).float()
    assert float((a - b).abs().max() / a.abs().max()) < 2e-2
    rmse = (a - ref).pow(2).mean().sqrt() / ref.abs().mean()
    assert float(rmse) < 0.1
    gs = cudagraph.GraphedSampler(m4, x, 10)
    g = gs.run(x).float()
    assert float((g - a).abs().max()) == 0.0
