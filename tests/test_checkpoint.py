"""Checkpoints: exact resume, legacy migration, failure safety, and interchange with the reference.

The interchange tests run the installed reference (``baseline/_ref``) in a
subprocess (its package is also called ``st``) and skip when it is absent.
"""
import json
import os
import subprocess
import sys
from pathlib import Path

import pytest
import torch

from exploration_b200 import ModelConfig, build_model, load_model
from exploration_b200.parallel.context import ParallelContext
from exploration_b200.runtime import checkpoint, faults
from exploration_b200.runtime.optim import FusedAdamW

ROOT = Path(__file__).resolve().parents[1]
REFERENCE = ROOT / "baseline" / "_ref"
WORKER = Path(__file__).with_name("ref_interchange_worker.py")
CONFIGS = {
    "stack": ModelConfig(model="stack", vocab_size=31, dim=16, heads=2, block_size=4, topk=64, arch="Lx2,(G)x2"),
    "baseline": ModelConfig(model="baseline", vocab_size=31, dim=16, heads=2, layers=2),
}


def _batch(seed=3, n=24):
    g = torch.Generator().manual_seed(seed)
    return {"ids": torch.randint(31, (2, n), generator=g), "targets": torch.randint(31, (2, n), generator=g)}


def _step(model, optimizer, batch):
    optimizer.zero_grad(set_to_none=True)
    result = model(batch["ids"], targets=batch["targets"])
    loss = result["loss_sum"] / result["count"]
    loss.backward()
    optimizer.step()
    return loss.detach()


def _save(path, model, optimizer, config, generator):
    checkpoint.save(path, model, optimizer, {"model": config.to_dict(), "runtime": {}}, 0, generator,
                    ParallelContext())


def test_resume_continues_bit_for_bit(tmp_path):
    torch.manual_seed(11)
    config = CONFIGS["stack"]
    model = build_model(config, execution={"backend": "torch", "encoder_chunk": 8})
    optimizer = FusedAdamW(model.parameters(), lr=1e-3)
    generator = torch.Generator().manual_seed(4)
    _step(model, optimizer, {"ids": torch.randint(31, (2, 17), generator=generator),
                             "targets": torch.randint(31, (2, 17), generator=generator)})
    path = tmp_path / "deep" / "run.pt"
    _save(path, model, optimizer, config, generator)
    batch = {"ids": torch.randint(31, (2, 17), generator=generator),
             "targets": torch.randint(31, (2, 17), generator=generator)}
    want_loss = _step(model, optimizer, batch)

    ck = checkpoint.load(path)
    assert ck["format_version"] == 2 and ck["topology"] == {"world_size": 1, "cp_size": 1}
    assert ck["model"]["embedding.weight"].data_ptr() == ck["model"]["lm_head.weight"].data_ptr()
    resumed = build_model(checkpoint.model_config(ck), execution={"backend": "torch", "encoder_chunk": 8})
    resumed.load_state_dict(ck["model"])
    resumed_opt = FusedAdamW(resumed.parameters(), lr=1e-3)
    resumed_opt.load_state_dict(ck["opt"])
    resumed_gen = torch.Generator()
    checkpoint.restore_rng(ck["rng_by_rank"][0], resumed_gen)
    again = {"ids": torch.randint(31, (2, 17), generator=resumed_gen),
             "targets": torch.randint(31, (2, 17), generator=resumed_gen)}
    assert torch.equal(again["ids"], batch["ids"])
    assert torch.equal(_step(resumed, resumed_opt, again), want_loss)
    for a, b in zip(model.parameters(), resumed.parameters()):
        assert torch.equal(a, b)
    assert sorted(p.name for p in path.parent.iterdir()) == ["run.pt"]


def test_legacy_arguments_are_migrated():
    stack = checkpoint.model_config({"args": {"d": 32, "b": 8, "heads": 4, "arch": "L,G", "task": "lm",
                                              "read_m": 4}})
    assert stack == {"vocab_size": 256, "dim": 32, "heads": 4, "ffn_ratio": 4, "block_size": 8, "topk": 4,
                     "arch": "L,G"}
    base = checkpoint.model_config({"args": {"model": "baseline", "layers": 5}})
    assert base["model"] == "baseline" and base["layers"] == 5 and base["vocab_size"] == 128


def test_a_failed_save_leaves_nothing_behind(tmp_path, monkeypatch):
    model = build_model(CONFIGS["baseline"])
    monkeypatch.setenv("EB200_FAULT", "checkpoint_write")
    faults.reset()
    with pytest.raises(RuntimeError, match="injected fault"):
        _save(tmp_path / "c.pt", model, torch.optim.AdamW(model.parameters()), CONFIGS["baseline"],
              torch.Generator())
    assert list(tmp_path.iterdir()) == []


def _reference(*args):
    if not (REFERENCE / "st" / "__init__.py").exists():
        pytest.skip("the reference is not installed in baseline/_ref")
    env = dict(os.environ, PYTHONPATH=str(REFERENCE))
    proc = subprocess.run([sys.executable, str(WORKER), *map(str, args)], capture_output=True, text=True, env=env,
                          cwd=args[1].parent, timeout=600)
    assert proc.returncode == 0, proc.stdout[-2000:] + proc.stderr[-3000:]


@pytest.mark.parametrize("kind", ["stack", "baseline"])
def test_reference_loads_our_checkpoint_and_resumes_its_optimizer(tmp_path, kind):
    torch.manual_seed(21)
    config = CONFIGS[kind]
    model = build_model(config, execution={"backend": "torch"}, dtype=torch.float64)
    optimizer = FusedAdamW(model.parameters(), lr=1e-3)
    batch = _batch()
    _step(model, optimizer, batch)
    path = tmp_path / "ours.pt"
    _save(path, model, optimizer, config, torch.Generator().manual_seed(1))
    torch.save(batch, tmp_path / "batch.pt")
    _reference("load", path, tmp_path / "batch.pt", tmp_path / "ref.pt")
    theirs = torch.load(tmp_path / "ref.pt")
    assert str(REFERENCE) in theirs["module"]
    model.eval()
    with torch.no_grad():
        torch.testing.assert_close(model(batch["ids"]), theirs["logits"], rtol=1e-5, atol=1e-6)
    model.train()
    _step(model, optimizer, batch)                     # the step the reference took after loading
    for name, value in model.named_parameters():
        torch.testing.assert_close(value.detach(), theirs["params"][name], rtol=1e-7, atol=1e-9, msg=name)


@pytest.mark.parametrize("kind", ["stack", "baseline"])
def test_we_load_a_reference_checkpoint(tmp_path, kind):
    config = CONFIGS[kind]
    (tmp_path / "config.json").write_text(json.dumps({"model": config.to_dict(), "runtime": {}}))
    batch = _batch(seed=8)
    torch.save(batch, tmp_path / "batch.pt")
    _reference("save", tmp_path / "theirs.pt", tmp_path / "config.json", tmp_path / "batch.pt", tmp_path / "ref.pt")
    theirs = torch.load(tmp_path / "ref.pt")
    model = load_model(tmp_path / "theirs.pt", dtype=torch.float64, execution={"backend": "torch"})
    with torch.no_grad():
        torch.testing.assert_close(model(batch["ids"]), theirs["logits"], rtol=1e-5, atol=1e-6)
    ck = checkpoint.load(tmp_path / "theirs.pt")
    optimizer = FusedAdamW(model.parameters(), lr=1e-3)
    optimizer.load_state_dict(ck["opt"])               # torch.optim.AdamW state fits the fused optimizer
    assert ck["step"] == 0 and len(ck["rng_by_rank"]) == 1
