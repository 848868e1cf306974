"""Subprocess side of the checkpoint interchange test: runs the *reference* framework.

Started with ``PYTHONPATH`` pointing at the installed reference (``baseline/_ref``)
and a working directory outside this repository, so ``import st`` is the
reference package. Usage::

    python ref_interchange_worker.py load  <checkpoint> <batch.pt> <out.pt>
    python ref_interchange_worker.py save  <checkpoint> <config.json> <batch.pt> <out.pt>

``load``: the reference's ``load_model`` reads a checkpoint written by this
repository; the worker records its logits on the batch, then restores the
optimizer state into ``torch.optim.AdamW`` and records the parameters after
one training step on the batch. ``save``: the reference builds the model of
``config.json``, takes one AdamW step, writes a checkpoint with its own
``checkpoint.save`` and records its logits.
"""
import json
import sys

import torch


def one_step(model, optimizer, batch):
    ids, targets = batch["ids"], batch["targets"]
    optimizer.zero_grad(set_to_none=True)
    result = model(ids, targets=targets)
    (result["loss_sum"] / result["count"]).backward()
    optimizer.step()


def main():
    import st  # the reference package
    from st.api import build_model, load_model
    from st.runtime import checkpoint
    from st.runtime.parallel import ParallelContext

    torch.set_default_dtype(torch.float64)
    mode = sys.argv[1]
    if mode == "load":
        path, batch_path, out = sys.argv[2:5]
        batch = torch.load(batch_path)
        model = load_model(path, dtype=torch.float64)
        with torch.no_grad():
            logits = model(batch["ids"])
        state = checkpoint.load(path)
        model.train()
        optimizer = torch.optim.AdamW(model.parameters(), lr=1e-3)
        optimizer.load_state_dict(state["opt"])
        one_step(model, optimizer, batch)
        torch.save({"logits": logits, "params": {k: v.detach() for k, v in model.named_parameters()},
                    "step": state["step"], "module": st.__file__}, out)
    elif mode == "save":
        path, config_path, batch_path, out = sys.argv[2:6]
        config = json.loads(open(config_path).read())
        batch = torch.load(batch_path)
        torch.manual_seed(5)
        model = build_model(config["model"], dtype=torch.float64)
        optimizer = torch.optim.AdamW(model.parameters(), lr=1e-3)
        one_step(model, optimizer, batch)
        checkpoint.save(path, model, optimizer, config, 0, torch.Generator().manual_seed(9), ParallelContext())
        model.eval()
        with torch.no_grad():
            logits = model(batch["ids"])
        torch.save({"logits": logits, "module": st.__file__}, out)
    else:
        raise SystemExit(f"unknown mode {mode}")


if __name__ == "__main__":
    main()
