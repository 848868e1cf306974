"""Recipes and helpers that run without a GPU: script syntax, the matrix report, heap sizing."""
import json
import subprocess
from pathlib import Path

import pytest

from exploration_b200 import build_model
from exploration_b200.parallel.context import ParallelContext

ROOT = Path(__file__).resolve().parents[1]
SCRIPTS = sorted((ROOT / "exploration_b200" / "recipes").rglob("*.sh"))


@pytest.mark.parametrize("script", SCRIPTS, ids=lambda p: p.name)
def test_recipe_parses(script):
    assert subprocess.run(["bash", "-n", str(script)], capture_output=True).returncode == 0
    assert "shutdown" not in script.read_text()


def test_scaling_matrix_report(tmp_path, capsys):
    from exploration_b200.recipes.experiments import scaling_matrix_report as report
    for name, bpc in (("sc_l1g1", 1.5), ("sc_l8g1", 1.2), ("sc_l1g1_base", 1.6)):
        (tmp_path / f"{name}.jsonl").write_text(json.dumps({"event": "eval", "length": 4096, "bpc": bpc}) + "\n")
    report.main(["--runs", str(tmp_path)])
    out = capsys.readouterr().out
    assert "1.5000" in out and "1.2000" in out and "L1 -> L8" in out


def test_fused_heap_sized_from_the_model():
    model = build_model({"model": "stack", **json.loads((ROOT / "configs/stack_500m.json").read_text())["model"]},
                        device="meta")
    parallel = ParallelContext()
    parallel.cp_size = 2
    need = parallel.fused_heap_bytes(model, 1, 65536)
    slot = 65536 * (model.heads // 2 * model.hd) * 2          # one bf16 head-layout slot
    assert need >= 8 * slot and need > 512 << 20             # the 500m run at CP=2 needs more than the default
    parallel.cp_size = 8
    assert parallel.fused_heap_bytes(model, 1, 65536) < need
