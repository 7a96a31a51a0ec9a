"""The matrix driver end to end on one GPU: a small custom shape over two EP
sizes and both reference routes, every case timed, checked and rendered."""
from __future__ import annotations

import json

import pytest

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("layout", ["padded", "packed"])
def test_matrix_run_small(cuda_device, tmp_path, layout):
    from sm90_fp8_wgrad import matrix as M

    rc = M.main(["run", "--models", "", "--model-spec", "small:16:2:512:256", "--ep", "1,4", "--route", "both",
                 "--tokens-list", "1000,3k", "--warmup-iters", "1", "--active-iters", "2", "--layout", layout,
                 "--output-dir", str(tmp_path)])
    assert rc == 0
    rows = [json.loads(x) for x in (tmp_path / "results.jsonl").read_text().splitlines()]
    assert len(rows) == 8
    for r in rows:
        assert r["passed"] and r["calc_diff"] <= 1e-5 and r["step_ms"] > 0
        assert len(r["ranks"]) == r["ep"]
        assert sum(p["valid_rows"] for p in r["ranks"]) == r["tokens"] * 2
    md = (tmp_path / "results.md").read_text()
    assert "## small (E=16, top-2, H=512, I=256)" in md
