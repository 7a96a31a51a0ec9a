"""Host logic of the model-shape matrix driver (no GPU): token parsing, case
enumeration, EP sharding of one global routing, the reference's EP proxy
sizes, Markdown rendering and the dry-run CLI."""
from __future__ import annotations

import json

import pytest

from sm90_fp8_wgrad import matrix as M


def test_parse_token_count():
    assert M.parse_token_count("4096") == 4096
    assert M.parse_token_count("4k") == 4096
    assert M.parse_token_count("32Ki") == 32768
    assert M.parse_token_count("16_384") == 16384
    with pytest.raises(RuntimeError):
        M.parse_token_count("0")
    with pytest.raises(RuntimeError):
        M.parse_token_count("")


def test_enumerate_cases_and_models():
    models = M.parse_models("all")
    assert models == ["qwen3_30b", "deepseek_v3", "minimax_m3", "qwen3_5_397b_a17b"]
    cases = M.enumerate_cases(["deepseek_v3"], [4096, 32768], [1, 8], ["balanced", "skewed"])
    assert len(cases) == 8 and cases[0] == M.Case("deepseek_v3", 4096, 1, "balanced")
    with pytest.raises(RuntimeError, match="does not divide"):
        M.enumerate_cases(["qwen3_30b"], [4096], [3], ["balanced"])
    with pytest.raises(RuntimeError, match="unknown model"):
        M.parse_models("gpt5")


def test_model_spec_parsing():
    name, spec = M.parse_model_spec("tiny:8:2:256:128")
    assert name == "tiny" and spec == ("tiny", 8, 2, 256, 128)
    with pytest.raises(RuntimeError):
        M.parse_model_spec("tiny:8:9:256:128")


@pytest.mark.parametrize("route", ["balanced", "skewed", "uniform", "zipf"])
def test_shard_mode_partitions_one_global_routing(route):
    case = M.Case("qwen3_30b", 2048, 4, route)
    probs = M.rank_problems(case, "shard", seed=3)
    assert len(probs) == 4
    routing = probs[0][0]
    assert all(p[0] is routing for p in probs)                 # one global routing
    spans = [p[1] for p in probs]
    assert spans == [(0, 32), (32, 64), (64, 96), (96, 128)]
    rows = sum(sum(routing.counts[a:b]) for a, b in spans)
    assert rows == 2048 * 8 == routing.valid_rows


def test_proxy_modes_follow_reference_sizes():
    case = M.Case("deepseek_v3", 4096, 8, "balanced")
    (r_real, span_real, t_real), = M.rank_problems(case, "proxy-real", seed=0)
    (r_stress, _, t_stress), = M.rank_problems(case, "proxy-stress", seed=0)
    assert span_real == (0, 32) and r_real.experts == 32
    assert t_real == 4096 and r_real.valid_rows == 4096 * 8
    assert t_stress == 4096 * 8 and r_stress.valid_rows == 4096 * 8 * 8


def _row(**kw):
    row = {"model": "deepseek_v3", "model_name": "DeepSeek-V3", "experts": 256, "top_k": 8, "hidden": 7168,
           "intermediate": 2048, "tokens": 32768, "ep": 1, "ep_mode": "shard", "route": "balanced",
           "layout": "padded", "tuned_config": "default", "seed": 1234, "step_ms": 19.0,
           "per_gpu_tflops": 1215.3, "pct_fp8_peak": 37.1, "slowest_rank_hbm_gbs": 1480.0, "imbalance": 1.0,
           "calc_diff": 2.4e-7, "diff_gate": 1e-3, "empty_experts_zero": True, "passed": True}
    row.update(kw)
    return row


def test_render_markdown_tables(tmp_path):
    rows = [_row(), _row(ep=8, step_ms=2.5, imbalance=1.07), _row(route="skewed", passed=False, calc_diff=0.5),
            _row(model="qwen3_30b", model_name="Qwen3-30B-A3B", experts=128, hidden=2048, intermediate=768)]
    md = M.render_markdown(rows)
    assert "## DeepSeek-V3 (E=256, top-8, H=7168, I=2048)" in md
    assert "## Qwen3-30B-A3B" in md
    assert "| balanced | 8 | 32k | 2.500 |" in md
    assert "| NO |" in md and "| yes |" in md
    p = tmp_path / "results.jsonl"
    p.write_text("\n".join(json.dumps(r) for r in rows) + "\n")
    out = tmp_path / "r.md"
    assert M.main(["render", str(p), "-o", str(out)]) == 0
    assert out.read_text() == md
    assert "(no results)" in M.render_markdown([])


def test_dry_run_lists_cases(capsys):
    assert M.main(["run", "--models", "qwen3_30b", "--ep", "1,8", "--route", "both", "--tokens-list", "4k,8k",
                   "--dry-run"]) == 0
    lines = [json.loads(x) for x in capsys.readouterr().out.splitlines()]
    assert len(lines) == 8
    assert {(c["ep"], c["route"], c["tokens"]) for c in lines} == {
        (e, r, t) for e in (1, 8) for r in ("balanced", "skewed") for t in (4096, 8192)}
