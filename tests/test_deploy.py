"""Deploy-compiler search on this package (kernel/compiler.py:97-172,
kernel/measure_table.py:35-61): the Pareto / budget decision logic on CPU
with the reference's own hand-made cases (kernel/selfcheck.py:62-81), and
one search on a B200."""
import pytest

from embodied_efficiency_b200.deploy import OBJECTIVES, make_row, pareto, pick_config


def test_pareto_and_budget_pick():
    rows = [
        {"precision": "bf16", "ms_per_action": 0.8, "weight_mb": 51, "rmse": 0.000, "staleness": 0},
        {"precision": "int8", "ms_per_action": 4.5, "weight_mb": 26, "rmse": 0.003, "staleness": 0},
        {"precision": "int4", "ms_per_action": 6.2, "weight_mb": 13, "rmse": 0.040, "staleness": 0},
        {"precision": "int8", "ms_per_action": 9.0, "weight_mb": 26, "rmse": 0.250, "staleness": 0},
    ]
    pf = pareto(rows)
    assert len(pf) == 3 and rows[3] not in pf
    assert pick_config(rows, {"objective": "ms_per_action", "max_rmse": 0.05})["precision"] == "bf16"
    assert pick_config(rows, {"objective": "weight_mb", "max_rmse": 0.05})["precision"] == "int4"
    assert pick_config(rows, {"max_weight_mb": 5}) is None
    stale = [{"precision": "bf16", "ms_per_action": 0.5, "weight_mb": 51, "rmse": 0.0, "staleness": 49},
             {"precision": "bf16", "ms_per_action": 6.0, "weight_mb": 51, "rmse": 0.0, "staleness": 0}]
    assert pick_config(stale, {"objective": "ms_per_action", "max_staleness": 0})["staleness"] == 0


def test_row_schema_and_exec_horizon_arithmetic():
    r = make_row("int4", 10, True, 12, 3.0, 31.1234, 0.04321, "plain")
    assert r == {"precision": "int4", "steps": 10, "graph": True, "exec_horizon": 12, "mode": "plain",
                 "call_ms": 3.0, "ms_per_action": 0.25, "weight_mb": 31.12, "rmse": 0.0432, "staleness": 11}
    assert set(OBJECTIVES) <= set(r)


@pytest.mark.gpu
def test_search_on_the_fused_sampler(cuda):
    """A full lever search at d_model 256: every precision x steps x graph x
    exec-horizon row plus the speculative rows, fidelity ordered as the
    quantisation depth, the full-step bf16 row exact, int4 below bf16 in
    footprint."""
    from embodied_efficiency_b200.deploy import search
    res = search(d_model=256, iters=5)
    rows = res["rows"]
    plain = [r for r in rows if r["mode"] == "plain"]
    assert len(plain) == 3 * 3 * 2 * 3
    assert len(rows) - len(plain) == 3 and all(r["mode"].startswith("spec(") for r in rows if r not in plain)
    full = {r["precision"]: r for r in plain if r["steps"] == 10 and r["graph"] and r["exec_horizon"] == 1}
    assert full["bf16"]["rmse"] == 0.0
    assert full["int8"]["rmse"] < 0.01 and full["int4"]["rmse"] < 0.10
    assert full["int4"]["weight_mb"] < full["int8"]["weight_mb"] < full["bf16"]["weight_mb"]
    assert all(r["call_ms"] > 0 for r in rows)
    assert pick_config(rows, {"objective": "ms_per_action", "max_rmse": 0.05, "max_staleness": 0}) is not None
