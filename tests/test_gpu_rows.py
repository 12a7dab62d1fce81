"""GPU parity of the layer-by-layer path's row kernels (ee_time_embed,
ee_expert_head, ee_euler_step) against the torch ops they replace
(kernel/flow_expert.py:38-48, :119-121, :133-136), computed in fp32 where the
reference rounds once: time embedding within one bf16 ulp of
timestep_embedding(t).to(bf16); the head within 1e-2 of max|ref| of the fp32
in_proj + bias (rounded) + temb; the Euler step bit-exact."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_time_embed_matches_timestep_embedding(cuda, dtype):
    from embodied_efficiency_b200.expert import _time_embedding_act, timestep_embedding
    t = (torch.arange(0, 11, device=cuda, dtype=torch.float32) / 10).to(dtype)
    for d in (256, 1024, 2048):
        got = _time_embedding_act(t, d, dtype).float()
        ref = timestep_embedding(t, d).to(dtype).float()
        ulp = 2.0 ** -7 if dtype == torch.bfloat16 else 2.0 ** -10
        assert (got - ref).abs().max().item() <= ulp, d


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("b,h,a,d", [(1, 50, 32, 1024), (256, 50, 32, 1024), (3, 7, 8, 256), (2, 50, 64, 2048)])
def test_expert_head_matches_in_proj_plus_temb(cuda, dtype, b, h, a, d):
    from embodied_efficiency_b200 import _lib
    g = torch.Generator(device="cpu").manual_seed(b * 31 + a)
    x_act = torch.randn(b, h, a, generator=g).to(dtype).to(cuda)
    w = (torch.randn(d, a, generator=g) * 0.2).to(dtype).to(cuda)
    bias = (torch.randn(d, generator=g) * 0.1).to(dtype).to(cuda)
    temb = torch.randn(b, d, generator=g).to(dtype).to(cuda)
    out = torch.empty(b, h, d, device=cuda, dtype=dtype)
    _lib.check(_lib.load().ee_expert_head(x_act.data_ptr(), w.data_ptr(), bias.data_ptr(), temb.data_ptr(),
                                          out.data_ptr(), b * h, a, d, h, d, _lib.act_code(dtype),
                                          _lib.stream_ptr(cuda)), "ee_expert_head")
    lin = (x_act.float() @ w.float().t() + bias.float()).to(dtype)
    ref = (lin.float() + temb.float()[:, None, :]).to(dtype).float()
    err = (out.float() - ref).abs().max().item() / ref.abs().max().item()
    assert err <= 1e-2, err
    # no bias: the same without the add
    _lib.check(_lib.load().ee_expert_head(x_act.data_ptr(), w.data_ptr(), None, temb.data_ptr(), out.data_ptr(),
                                          b * h, a, d, h, d, _lib.act_code(dtype), _lib.stream_ptr(cuda)),
               "ee_expert_head")
    ref0 = ((x_act.float() @ w.float().t()).to(dtype).float() + temb.float()[:, None, :]).to(dtype).float()
    assert (out.float() - ref0).abs().max().item() / ref0.abs().max().item() <= 1e-2


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("n_steps", [1, 3, 10])
def test_euler_step_bit_exact(cuda, dtype, n_steps):
    from embodied_efficiency_b200.expert import _euler_step
    g = torch.Generator(device="cpu").manual_seed(n_steps)
    x = torch.randn(5, 50, 32, generator=g).to(dtype).to(cuda)
    t = torch.zeros(5, device=cuda, dtype=dtype)
    xr, tr = x.clone(), t.clone()
    dt = 1.0 / n_steps
    for _ in range(n_steps):
        v = torch.randn(5, 50, 32, generator=g).to(dtype).to(cuda)
        x, t = _euler_step(x, v, t, dt)
        xr, tr = xr + v * dt, tr + dt
    assert torch.equal(x, xr) and torch.equal(t, tr)


def test_row_kernel_argument_errors(cuda):
    from embodied_efficiency_b200 import _lib
    lib = _lib.load()
    buf = torch.zeros(4096, device=cuda, dtype=torch.bfloat16)
    p = buf.data_ptr()
    assert lib.ee_time_embed(p, p, p, 2, 7, _lib.EE_BF16, None) != 0          # odd dim
    assert lib.ee_expert_head(p, p, None, p, p, 4, 12, 256, 1, 256, _lib.EE_BF16, None) != 0   # action_dim % 8
    assert lib.ee_expert_head(p, p, None, p, p, 4, 72, 256, 1, 256, _lib.EE_BF16, None) != 0   # action_dim > 64
    assert lib.ee_euler_step(p, p, None, 16, 0, 0.1, 99, None) != 0           # dtype
    assert lib.ee_euler_step(p, p, None, 0, 0, 0.1, _lib.EE_BF16, None) == 0  # empty
