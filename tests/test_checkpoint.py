"""Packed-weight checkpoints of quantized models (kernel/triton_gemm.py:177-178:
``weight`` and ``scales`` are registered buffers, so ``state_dict`` carries
the quantized form). CPU only: int8 modules quantize without a GPU.

A checkpoint round trip restores the packed buffers exactly, holds nothing
but the reference's buffers (the dense weight copy that GEMMs of many tokens
run on is a cache, not state), and loading one bumps the buffers' versions,
which is what retires a cached dense copy made from the old weights."""
import io

import torch

from embodied_efficiency_b200 import quantize_model_triton
from embodied_efficiency_b200.expert import ActionExpert, ActionExpertConfig


def _model(seed):
    torch.manual_seed(seed)
    cfg = ActionExpertConfig(d_model=256, n_layers=2, n_heads=4, prefix_len=16)
    return quantize_model_triton(ActionExpert(cfg), bits=8)


def test_state_dict_round_trip_restores_packed_buffers():
    src, dst = _model(0), _model(1)
    sd = src.state_dict()
    buf = io.BytesIO()
    torch.save(sd, buf)
    buf.seek(0)
    loaded = torch.load(buf)
    versions = {k: v._version for k, v in dst.state_dict(keep_vars=True).items()}
    dst.load_state_dict(loaded)
    after = dst.state_dict(keep_vars=True)
    for k, v in sd.items():
        assert torch.equal(after[k], v), k
    q = dst.blocks[0].q_c
    assert type(q).__name__ == "TritonQuantLinear"
    assert q.weight.dtype == torch.int8 and q.scales.dtype == torch.float32
    # every quantized buffer was written in place: a cached dense copy keyed
    # on (storage, version) no longer matches
    for k in ("blocks.0.q_c.weight", "blocks.0.q_c.scales", "blocks.1.mlp.0.weight"):
        assert after[k]._version > versions[k], k


def test_checkpoint_holds_only_the_reference_buffers():
    m = _model(2)
    q = m.blocks[0].qkv
    q.__dict__["_dense"] = (None, torch.zeros(1))  # a stale cache entry is not state
    keys = [k for k in m.state_dict() if k.startswith("blocks.0.qkv.")]
    assert sorted(keys) == ["blocks.0.qkv.bias", "blocks.0.qkv.scales", "blocks.0.qkv.weight"]
