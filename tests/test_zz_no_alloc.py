"""ee_flow_sample_noalloc: the sampler for callers that cannot allocate device
memory (hard-real-time control loops, hosts that own all device memory behind
an FFI), with its workspace in a fixed array inside the library. Checked
through the C ABI against ee_flow_sample with a caller workspace, on two calls
in a row. This file sorts last so that a stop-at-first-failure run has run
every other test before it."""
import ctypes

import pytest
import torch

from oracle import sampler as OS

pytestmark = pytest.mark.gpu
ACTION_TOL = 0.05  # the sampler tests' action-error tolerance


def _plan(cuda, batch=1, kw=None):
    from embodied_efficiency_b200 import ActionExpert, ActionExpertConfig, quantize_model_triton, synth
    cfg = ActionExpertConfig(**(kw or dict(d_model=1024, n_layers=4, n_heads=16, prefix_len=256)))
    params, x0, prefix = synth.workload(cfg, seed=0, batch=batch)
    m = ActionExpert(cfg)
    m.load_state_dict(params)
    m = quantize_model_triton(m.to(cuda).bfloat16().eval(), bits=4)
    kv = m.encode(prefix.to(cuda))
    return m.plan(batch, kv), x0.to(cuda).bfloat16()


def test_noalloc_matches_workspace_entry_point(cuda):
    from embodied_efficiency_b200 import _lib
    lib = _lib.load()
    plan, x = _plan(cuda)
    ref = plan.run(x, 10)
    torch.cuda.synchronize()
    for call in range(2):  # two calls in a row share the static workspace
        out = torch.empty_like(x)
        rc = lib.ee_flow_sample_noalloc(ctypes.byref(plan.ex), x.data_ptr(), None, out.data_ptr(),
                                        10, _lib.EE_MODE_EULER, _lib.stream_ptr(cuda))
        assert rc == 0, _lib.strerror(rc)
        torch.cuda.synchronize()
        err = OS.action_error(out.float().cpu(), ref.float().cpu())
        assert err <= ACTION_TOL, (call, err)
        assert torch.equal(out, ref), f"call {call}: differs from ee_flow_sample"


def test_noalloc_rejects_oversized_workspace(cuda):
    from embodied_efficiency_b200 import _lib
    lib = _lib.load()
    plan, x = _plan(cuda, batch=16, kw=dict(d_model=512, n_layers=2, n_heads=8, prefix_len=32))
    need = lib.ee_flow_sample_workspace_bytes(ctypes.byref(plan.ex), 10)
    assert need > 4 << 20
    out = torch.zeros_like(x)
    rc = lib.ee_flow_sample_noalloc(ctypes.byref(plan.ex), x.data_ptr(), None, out.data_ptr(), 10,
                                    _lib.EE_MODE_EULER, _lib.stream_ptr(cuda))
    assert rc == 5  # EE_ERR_WORKSPACE: nothing was launched
    torch.cuda.synchronize()
    assert out.abs().sum().item() == 0.0
