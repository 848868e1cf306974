"""Summary of the L x G scaling matrix (``runs/sc_*.jsonl`` from scaling_matrix.sh).

``python -m exploration_b200.recipes.experiments.scaling_matrix_report [--runs runs]``

For the training length (4096) and the zero-shot lengths (16384, 65536) it
prints the Stack bpc matrix, the matched-baseline bpc matrix, their ratio
(baseline / Stack) and the marginal gains along each side (L1 -> L8 at fixed
G, G1 -> G4 at fixed L). An eval record is a JSON line with ``event == "eval"``,
``length`` and ``bpc``; the last record per length wins. (Counterpart of the
reference's scripts/experiments/scaling_matrix_report.py.)
"""
from __future__ import annotations

import argparse
import json
from pathlib import Path

LENGTHS = (4096, 16384, 65536)
L_SIDE = (1, 2, 4, 8)
G_SIDE = (1, 2, 4)


def bpc_by_length(path: Path) -> dict[int, float]:
    found: dict[int, float] = {}
    if not path.exists():
        return found
    for line in path.read_text().splitlines():
        try:
            record = json.loads(line)
        except json.JSONDecodeError:
            continue
        if record.get("event") == "eval" and "bpc" in record and "length" in record:
            found[int(record["length"])] = float(record["bpc"])
    return found


def table(title: str, value) -> str:
    rows = [f"\n{title} (rows: G, columns: L)", "     " + "".join(f"{'L=' + str(l):>9}" for l in L_SIDE)]
    for g in G_SIDE:
        cells = []
        for l in L_SIDE:
            v = value(l, g)
            cells.append(f"{v:9.4f}" if v is not None else f"{'-':>9}")
        rows.append(f"G={g:<3}" + "".join(cells))
    return "\n".join(rows)


def main(argv=None) -> None:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--runs", default="runs")
    args = p.parse_args(argv)
    runs = Path(args.runs)
    stack = {(l, g): bpc_by_length(runs / f"sc_l{l}g{g}.jsonl") for l in L_SIDE for g in G_SIDE}
    base = {(l, g): bpc_by_length(runs / f"sc_l{l}g{g}_base.jsonl") for l in L_SIDE for g in G_SIDE}
    for n in LENGTHS:
        print(f"\n===== length {n} =====")
        print(table("Stack bpc", lambda l, g: stack[l, g].get(n)))
        print(table("baseline bpc", lambda l, g: base[l, g].get(n)))

        def ratio(l, g):
            s, b = stack[l, g].get(n), base[l, g].get(n)
            return b / s if s and b else None
        print(table("baseline / Stack", ratio))
        for g in G_SIDE:
            a, b = stack[1, g].get(n), stack[8, g].get(n)
            if a and b:
                print(f"write side G={g}: L1 -> L8 bpc {a:.4f} -> {b:.4f} ({(a - b) / a:+.1%})")
        for l in L_SIDE:
            a, b = stack[l, 1].get(n), stack[l, 4].get(n)
            if a and b:
                print(f"read side L={l}: G1 -> G4 bpc {a:.4f} -> {b:.4f} ({(a - b) / a:+.1%})")


if __name__ == "__main__":
    main()
