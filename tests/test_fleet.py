"""Fleet mode host logic (sharding, chunking, result assembly) on CPU with
gloo ranks, and one GPU run against single-request sampler calls."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from embodied_efficiency_b200.fleet import FleetSampler, chunk_bounds, gather_results, shard_bounds


@pytest.mark.parametrize("n,world", [(256, 1), (256, 2), (256, 8), (7, 3), (2, 4), (0, 2)])
def test_shard_bounds_cover_once(n, world):
    seen = []
    prev_hi = 0
    for r in range(world):
        lo, hi = shard_bounds(n, r, world)
        assert lo == prev_hi and hi >= lo
        assert hi - lo in (n // world, n // world + 1)
        seen += list(range(lo, hi))
        prev_hi = hi
    assert seen == list(range(n))


def test_shard_and_chunk_errors():
    with pytest.raises(ValueError):
        shard_bounds(4, 2, 2)
    with pytest.raises(ValueError):
        chunk_bounds(0, 4, 0)
    assert chunk_bounds(3, 10, 3) == [(3, 6), (6, 9), (9, 10)]
    assert chunk_bounds(5, 5, 4) == []


class _Cfg:
    horizon, action_dim, prefix_len, d_model = 5, 4, 3, 8


def _request(i):
    g = torch.Generator().manual_seed(i)
    return torch.randn(1, _Cfg.prefix_len, _Cfg.d_model, generator=g), torch.randn(1, _Cfg.horizon, _Cfg.action_dim, generator=g)


def _fake_sample(pre, x0):
    # stands in for the sampler: any per-request function of (prefix, noise)
    return x0 * 0.5 + pre.mean(dim=(1, 2))[:, None, None]


def _worker(rank, world, port, n, chunk, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.distributed.init_process_group("gloo", rank=rank, world_size=world)
    try:
        fs = FleetSampler(n, rank, world, chunk=chunk, sample_fn=_fake_sample).stage(_request)
        shard = fs.run()
        assert shard.actions.shape[0] == shard.hi - shard.lo
        full = gather_results(shard, n)
        if rank == 0:
            q.put(full)
    finally:
        torch.distributed.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("n,chunk", [(11, 4), (8, 8)])
def test_fleet_gloo_two_ranks(n, chunk):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, n, chunk, q)) for r in range(2)]
    for p in procs:
        p.start()
    full = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    ref = torch.cat([_fake_sample(*_request(i)) for i in range(n)], 0)
    torch.testing.assert_close(full, ref)


def test_fleet_single_process_matches_per_request():
    fs = FleetSampler(9, 0, 1, chunk=4, sample_fn=_fake_sample).stage(_request)
    shard = fs.run()
    ref = torch.cat([_fake_sample(*_request(i)) for i in range(9)], 0)
    torch.testing.assert_close(shard.actions, ref)
    with pytest.raises(ValueError):
        FleetSampler(4, 0, 1)


@pytest.mark.gpu
def test_fleet_gpu_matches_single_calls(cuda):
    """Chunked fused launches give each request what its own batch-1 sampler
    call gives (same weights, prefix and noise)."""
    from embodied_efficiency_b200 import ActionExpert, ActionExpertConfig, flow_sample, quantize_model_triton, synth
    cfg = ActionExpertConfig(d_model=256, n_layers=2, n_heads=4, prefix_len=32)
    params, _, _ = synth.workload(cfg, seed=3)
    m = ActionExpert(cfg)
    m.load_state_dict(params)
    m = m.to(cuda).bfloat16().eval()
    quantize_model_triton(m, bits=4)
    req = lambda i: synth.fleet_request(cfg, i)  # noqa: E731
    fs = FleetSampler(6, 0, 1, chunk=4, expert=m, device=cuda).stage(req)
    got = fs.run().actions
    for i in range(6):
        pre, x0 = req(i)
        kv = m.encode(pre.to(cuda))
        one = flow_sample(m, x0.to(cuda).bfloat16(), 10, kv).float().cpu()
        err = (got[i:i + 1] - one).abs().max() / one.abs().max()
        assert err < 2e-2, (i, float(err))


@pytest.mark.gpu
@pytest.mark.parametrize("n,chunk", [(6, 4), (40, 40), (64, 32)])
def test_fleet_graphs_match_direct_calls(cuda, n, chunk):
    """Each chunk's call captured as a CUDA graph (fused launch for small
    chunks, the layer-by-layer path from 1024 tokens on) replays what the
    directly dispatched calls compute, fleet step after fleet step."""
    from embodied_efficiency_b200 import ActionExpert, ActionExpertConfig, quantize_model_triton, synth
    cfg = ActionExpertConfig(d_model=256, n_layers=2, n_heads=4, prefix_len=32)
    params, _, _ = synth.workload(cfg, seed=4)
    m = ActionExpert(cfg)
    m.load_state_dict(params)
    m = m.to(cuda).bfloat16().eval()
    quantize_model_triton(m, bits=4)
    req = lambda i: synth.fleet_request(cfg, i)  # noqa: E731
    direct = FleetSampler(n, 0, 1, chunk=chunk, expert=m, device=cuda, graphs=False).stage(req).run().actions
    fs = FleetSampler(n, 0, 1, chunk=chunk, expert=m, device=cuda).stage(req)
    assert fs._graphs is not None and len(fs._graphs) == len(chunk_bounds(0, n, chunk))
    for _ in range(2):
        got = fs.run().actions
        err = float((got - direct).abs().max() / direct.abs().max())
        print(f"fleet n={n} chunk={chunk}: graph vs direct max rel diff {err:.3e}")
        assert err < 2e-2
