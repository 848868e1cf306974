"""Command-line and public-API contract of this framework.

The option table in ``exploration_b200.cli`` is the single definition of
every flag, its group and the subcommands that hide it; these tests derive
their expectations from that table instead of listing flags by hand. Runs
go through ``main`` (the console entry point's body) on tiny CPU models.
The contract itself is the reference's (st/cli.py:16-209, tests/test_cli.py):
the same commands, precedence, legacy rejections and checkpoint migration.
"""
import contextlib
import io
import json
from pathlib import Path
from unittest.mock import patch

import pytest
import torch

from exploration_b200 import ExecutionConfig, ModelConfig, StackModel, build_model, load_model
from exploration_b200 import cli
from exploration_b200.runtime import checkpoint

CPU = ("--device", "cpu", "--backend", "torch", "--precision", "fp32")
TINY = ("--task", "random", "--vocab-size", "31", "--dim", "16", "--heads", "2", "--block-size", "4",
        "--arch", "L,G")
CONFIGS = Path(__file__).resolve().parents[1] / "configs"


def run(*argv):
    """``main(argv)`` with its JSON event lines captured: (return value, events)."""
    out = io.StringIO()
    with contextlib.redirect_stdout(out):
        result = cli.main(list(argv))
    return result, [json.loads(line) for line in out.getvalue().splitlines() if line.startswith("{")]


def help_text(command):
    out = io.StringIO()
    with contextlib.redirect_stdout(out), pytest.raises(SystemExit) as stop:
        cli.main([command, "--help"])
    assert stop.value.code == 0
    return out.getvalue()


# -- command surface --------------------------------------------------------

@pytest.mark.parametrize("command", ["plan", "train", "eval"])
def test_help_shows_exactly_the_options_the_table_makes_visible(command):
    text = help_text(command)
    for flag, group, kwargs in cli.OPTIONS:
        shown = cli._visible(command, group, cli._dest(flag, kwargs))
        # "--flag " or "--flag\n": avoid prefix matches such as --cache / --cache-dir.
        present = any(f"{flag}{end}" in text for end in (" ", "\n", ","))
        assert present == shown, (command, flag)


def test_bare_invocation_lists_every_command():
    out = io.StringIO()
    with contextlib.redirect_stdout(out):
        cli.main([])
    for command in cli.COMMANDS:
        assert command in out.getvalue()


def test_benchmark_and_validate_have_their_own_parsers():
    bench, valid = help_text("benchmark"), help_text("validate")
    assert "--compare" in bench and "--resume" not in bench
    assert "--suite" in valid and "--dim" not in valid
    for suite in ("reference", "resources", "cuda", "distributed"):
        assert suite in valid


def test_console_script_returns_nothing():
    with patch.object(cli, "main", return_value={"loss": 0.5}) as body:
        assert cli.entrypoint() is None
    body.assert_called_once_with()


def test_reference_package_name_resolves_to_these_modules():
    import st
    import st.attention
    import st.blocks
    import st.stack_model
    from exploration_b200.data import synthetic
    from exploration_b200.models import blocks, stack
    from exploration_b200.ops import attention
    assert (st.blocks, st.stack_model.StackModel, st.attention.dense_attention) == \
        (blocks, stack.StackModel, attention.dense_attention)
    assert st.data.Q == synthetic.Q == 31 and st.data.KEY == synthetic.KEY == 5


# -- JSON configs and precedence -------------------------------------------

@pytest.mark.parametrize("name", sorted(p.stem for p in CONFIGS.glob("*.json")))
def test_shipped_configs_parse_and_plan(name):
    args = cli.parse_args(["plan", "--config", str(CONFIGS / f"{name}.json")])
    assert args.dim > 0 and args.heads > 0 and args.dim % args.heads == 0


@pytest.mark.parametrize("runtime", [{"precision": "fp16"}, {"batch_size": 2.5}, {"checkpoint_chunks": "no"},
                                     {"command": "train"}, {"not_a_flag": 1}])
def test_json_values_are_checked_like_flags(tmp_path, runtime):
    path = tmp_path / "bad.json"
    path.write_text(json.dumps({"runtime": runtime}))
    with contextlib.redirect_stderr(io.StringIO()), pytest.raises((SystemExit, ValueError)):
        cli.parse_args(["plan", "--config", str(path)])


def test_flag_beats_json_beats_default(tmp_path):
    path = tmp_path / "cfg.json"
    path.write_text(json.dumps({"model": {"dim": 48, "heads": 6}, "runtime": {"batch_size": 3}}))
    args = cli.parse_args(["plan", "--config", str(path), "--heads", "3"])
    assert (args.dim, args.heads, args.batch_size, args.block_size) == (48, 3, 3, 16)
    out = io.StringIO()
    with contextlib.redirect_stdout(out):
        cli.main(["plan", "--config", str(path), "--heads", "3"])
    planned = json.loads(out.getvalue())["model"]
    assert (planned["heads"], planned["dim"]) == (3, 48)


@pytest.mark.parametrize("argv", [["train", "--length", str((1 << 16) + 1)], ["train", "--topk", "0"],
                                  ["train", "--stop-exact", "0.5"], ["train", "--ema", "0.99"],
                                  ["train", "--task", "tokens", "--eval-every", "5"]])
def test_out_of_range_and_retired_flags_fail(argv):
    with contextlib.redirect_stderr(io.StringIO()), pytest.raises(SystemExit):
        cli.parse_args(argv)


# -- public API and checkpoints ---------------------------------------------

def test_build_model_then_load_a_legacy_args_checkpoint(tmp_path):
    model = build_model(ModelConfig(vocab_size=128, dim=24, heads=3, block_size=4, arch="L,G"),
                        execution=ExecutionConfig(backend="torch", encoder_chunk=8))
    assert isinstance(model, StackModel)
    # Legacy files carry only the old argument names; the vocabulary follows the task (128).
    legacy = {"model": model.state_dict(),
              "args": {"model": "stack", "d": 24, "heads": 3, "b": 4, "arch": "L,G", "task": "passkey"}}
    torch.save(legacy, tmp_path / "old.pt")
    loaded = load_model(tmp_path / "old.pt", topk=3, execution=ExecutionConfig(backend="torch", encoder_chunk=8))
    assert (loaded.topk, loaded.dim, loaded.training) == (3, 24, False)
    for (name, a), b in zip(model.state_dict().items(), loaded.state_dict().values()):
        assert torch.equal(a, b), name


def test_training_loss_ignores_the_inference_topk():
    torch.manual_seed(3)
    execution = ExecutionConfig(backend="torch", encoder_chunk=8)
    models = [build_model(ModelConfig(vocab_size=31, dim=16, heads=2, block_size=4, topk=k), execution=execution)
              for k in (1, 2, 50)]
    for other in models[1:]:
        other.load_state_dict(models[0].state_dict())
    ids = torch.randint(31, (2, 19))
    targets = torch.randint(31, ids.shape)
    losses = [m(ids, targets=targets)["loss_sum"] for m in models]
    assert all(torch.equal(losses[0], x) for x in losses[1:])


# -- one driver for train and eval ------------------------------------------

@pytest.mark.parametrize("kind", ["stack", "baseline"])
def test_train_then_eval_a_checkpoint_of_either_model(tmp_path, kind):
    ck = tmp_path / f"{kind}.pt"
    _, events = run("train", "--model", kind, *TINY, "--layers", "1", "--length", "17", "--batch-size", "2",
                    "--encoder-chunk", "8", "--query-chunk", "3", *CPU, "--steps", "2", "--grad-accum", "2",
                    "--eval-every", "1", "--log-every", "1", "--save", str(ck))
    assert {"train", "eval"} <= {e.get("event") for e in events}
    saved = checkpoint.load(ck)
    assert saved["config"]["model"]["model"] == kind and saved["step"] == 1 and "ema" not in saved
    result, _ = run("eval", "--resume", str(ck), "--task", "random", "--length", "23", "--eval-positions", "3",
                    "--cache", "cpu", *CPU)
    assert result["evaluated_tokens"] == 3 and torch.isfinite(torch.tensor(result["loss"]))


def test_stopped_run_resumes_onto_the_uninterrupted_weights(tmp_path):
    common = (*TINY, "--length", "17", "--batch-size", "2", "--encoder-chunk", "8", "--log-every", "1", *CPU)
    whole, piece = tmp_path / "whole.pt", tmp_path / "piece.pt"
    run("train", *common, "--steps", "3", "--save", str(whole))
    # --stop-exact 0 ends the run at its first periodic evaluation (after step 2 of 3).
    run("train", *common, "--steps", "3", "--save", str(piece), "--save-every", "1", "--stop-exact", "0",
        "--eval-every", "2")
    assert checkpoint.load(piece)["step"] == 1
    run("train", *common, "--steps", "3", "--save", str(piece), "--resume", str(piece))
    finished, reference = checkpoint.load(piece), checkpoint.load(whole)
    assert finished["step"] == reference["step"] == 2
    for name, value in reference["model"].items():
        assert torch.equal(finished["model"][name], value), name


def test_profile_flag_leaves_a_trace_and_a_summary(tmp_path):
    _, events = run("train", *TINY, "--length", "17", "--batch-size", "2", *CPU, "--steps", "6",
                    "--log-every", "100", "--save", "", "--profile", str(tmp_path / "trace"))
    profile = [e for e in events if e.get("event") == "profile"]
    assert len(profile) == 1 and Path(profile[0]["trace"]).exists() and profile[0]["top"]
