"""CLI and public API contract, including the reference's package name ``st``."""
import contextlib
import io
import json
from pathlib import Path
from unittest.mock import patch

import pytest
import torch

from exploration_b200 import ExecutionConfig, ModelConfig, StackModel, build_model, load_model
from exploration_b200.cli import entrypoint, main, parse_args
from exploration_b200.runtime import checkpoint

CPU = ["--device", "cpu", "--backend", "torch", "--precision", "fp32"]


def test_reference_module_aliases():
    import st.attention
    import st.blocks
    import st.stack_model
    from st import data
    from st.models import blocks, stack
    from st.ops import attention
    assert st.blocks is blocks
    assert st.stack_model.StackModel is stack.StackModel
    assert st.attention.dense_attention is attention.dense_attention
    assert data.Q == 31 and data.KEY == 5


def test_scoped_help_and_no_args():
    with contextlib.redirect_stdout(io.StringIO()) as out:
        main([])
    assert "benchmark" in out.getvalue()
    for command, present, absent in (("eval", "--cache", "--grad-accum"),
                                     ("plan", "--dim", "--eval-every"),
                                     ("benchmark", "--compare", "--resume")):
        with contextlib.redirect_stdout(io.StringIO()) as out, pytest.raises(SystemExit) as caught:
            main([command, "--help"])
        assert caught.value.code == 0
        assert present in out.getvalue() and absent not in out.getvalue()


def test_console_entrypoint_discards_result():
    with patch("exploration_b200.cli.main", return_value={"loss": 1.0}) as driver:
        assert entrypoint() is None
    driver.assert_called_once_with()


def test_json_defaults_are_validated(tmp_path):
    path = tmp_path / "config.json"
    for runtime in ({"precision": "fp64"}, {"batch_size": 1.5}, {"checkpoint_chunks": "false"},
                    {"command": "eval"}):
        path.write_text(json.dumps({"runtime": runtime}))
        with contextlib.redirect_stderr(io.StringIO()), pytest.raises((SystemExit, ValueError)):
            parse_args(["plan", "--config", str(path)])


def test_public_build_load_and_legacy_checkpoint(tmp_path):
    config = ModelConfig(vocab_size=128, dim=16, heads=2, block_size=4, arch="L,G")
    model = build_model(config, execution=ExecutionConfig(backend="torch", encoder_chunk=8))
    assert isinstance(model, StackModel)
    path = tmp_path / "legacy.pt"
    torch.save({"model": model.state_dict(), "args": {"model": "stack", "d": 16, "heads": 2, "b": 4,
                                                       "arch": "L,G", "task": "mqar", "read_m": 64}}, path)
    other = load_model(path, topk=2, execution=ExecutionConfig(backend="torch", encoder_chunk=8))
    assert other.topk == 2 and other.dim == 16 and not other.training
    for p, q in zip(model.parameters(), other.parameters()):
        torch.testing.assert_close(p, q, atol=0, rtol=0)


@pytest.mark.parametrize("kind", ["stack", "baseline"])
def test_train_eval_share_one_driver(tmp_path, kind):
    ck = str(tmp_path / "model.pt")
    common = ["--model", kind, "--task", "random", "--vocab-size", "31", "--dim", "16", "--heads", "2",
              "--block-size", "4", "--arch", "L,G", "--layers", "1", "--length", "17", "--batch-size",
              "2", "--encoder-chunk", "8", "--query-chunk", "3"]
    with contextlib.redirect_stdout(io.StringIO()):
        main(["train", *common, *CPU, "--steps", "2", "--grad-accum", "2", "--eval-every", "1",
              "--save", ck])
        result = main(["eval", "--resume", ck, "--task", "random", "--length", "23",
                       "--eval-positions", "3", "--cache", "cpu", *CPU])
    saved = checkpoint.load(ck)
    assert saved["config"]["model"]["model"] == kind
    assert saved["step"] == 1 and result["evaluated_tokens"] == 3
    assert torch.isfinite(torch.tensor(result["loss"]))


def test_exact_resume_continues_the_run(tmp_path):
    common = ["--task", "random", "--vocab-size", "31", "--dim", "16", "--heads", "2",
              "--block-size", "4", "--arch", "L,G", "--length", "17", "--batch-size", "2",
              "--encoder-chunk", "8", "--log-every", "1", *CPU]
    full, part = str(tmp_path / "full.pt"), str(tmp_path / "part.pt")
    with contextlib.redirect_stdout(io.StringIO()):
        main(["train", *common, "--steps", "3", "--save", full])
        main(["train", *common, "--steps", "3", "--save", part, "--save-every", "1",
              "--stop-exact", "0", "--eval-every", "2"])
    # The second run stopped early after step 2; resuming must land on the same weights.
    assert checkpoint.load(part)["step"] == 1
    with contextlib.redirect_stdout(io.StringIO()):
        main(["train", *common, "--steps", "3", "--save", part, "--resume", part])
    done, ref = checkpoint.load(part), checkpoint.load(full)
    assert done["step"] == ref["step"] == 2
    for name, value in ref["model"].items():
        torch.testing.assert_close(done["model"][name], value, atol=0, rtol=0, msg=name)


def test_config_round_trip_and_precedence(tmp_path):
    path = tmp_path / "config.json"
    path.write_text(json.dumps({"model": {"dim": 32, "heads": 4}, "runtime": {"batch_size": 2}}))
    args = parse_args(["plan", "--config", str(path), "--dim", "16"])
    assert args.dim == 16 and args.batch_size == 2
    with contextlib.redirect_stdout(io.StringIO()) as output:
        main(["plan", "--config", str(path), "--dim", "16"])
    assert json.loads(output.getvalue())["model"]["dim"] == 16


def test_dense_loss_does_not_depend_on_inference_topk():
    torch.manual_seed(14)
    execution = ExecutionConfig(backend="torch", encoder_chunk=8)
    small = build_model(ModelConfig(vocab_size=31, dim=16, heads=2, block_size=4, topk=1),
                        execution=execution)
    large = build_model(ModelConfig(vocab_size=31, dim=16, heads=2, block_size=4, topk=64),
                        execution=execution)
    large.load_state_dict(small.state_dict())
    ids = torch.randint(31, (1, 21))
    targets = torch.randint(31, ids.shape)
    torch.testing.assert_close(small(ids, targets=targets)["loss_sum"],
                               large(ids, targets=targets)["loss_sum"], atol=0, rtol=0)


def test_invalid_cli_and_legacy_flags_are_rejected():
    for argv in (["train", "--length", "65537"], ["train", "--topk", "0"],
                 ["train", "--stop-exact", ".99"], ["train", "--ema", ".9"],
                 ["train", "--task", "tokens", "--eval-every", "1"]):
        with contextlib.redirect_stderr(io.StringIO()), pytest.raises(SystemExit):
            parse_args(argv)


def test_reference_configs_parse():
    root = Path(__file__).resolve().parents[1] / "configs"
    for name in ("stack_2m", "stack_100m", "stack_500m", "baseline_2m"):
        args = parse_args(["plan", "--config", str(root / f"{name}.json")])
        assert args.dim > 0


def test_train_profile_writes_a_trace(tmp_path):
    out = io.StringIO()
    common = ["--task", "random", "--vocab-size", "31", "--dim", "16", "--heads", "2", "--block-size", "4",
              "--arch", "L,G", "--length", "17", "--batch-size", "2"]
    with contextlib.redirect_stdout(out):
        main(["train", *common, *CPU, "--steps", "6", "--log-every", "100", "--save", "",
              "--profile", str(tmp_path / "prof")])
    events = [json.loads(line) for line in out.getvalue().splitlines() if line.startswith("{")]
    profile = [e for e in events if e.get("event") == "profile"]
    assert profile and Path(profile[0]["trace"]).exists()
    assert profile[0]["top"]
