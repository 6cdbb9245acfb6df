"""Generates tests/golden/distributed.json from the reference's own sample
scheduling (xfold/distributed.py: work_indices, sample_seed) and its initial
noise draw for a diffusion sample (xfold/alphafold3.py:415-420: the global CPU
generator set from a generator seeded with sample_seed, then randn times the
first noise level).

Usage (from the repository root, with the reference checkout available):
    PYTHONPATH=<xfold checkout> python tests/golden/make_distributed_golden.py
"""

from __future__ import annotations

import json
from pathlib import Path

import torch

from xfold.distributed import sample_seed, work_indices

OUT = Path(__file__).resolve().parent / "distributed.json"


def main() -> None:
    cases = []
    for total, world, schedule, weights in [
        (5, 1, "cyclic", ()), (5, 2, "cyclic", ()), (5, 8, "cyclic", ()), (0, 3, "cyclic", ()),
        (5, 2, "block", ()), (7, 3, "block", ()), (2, 4, "block", ()),
        (10, 3, "weighted", (1, 2, 3)), (5, 2, "weighted", (0, 1)), (9, 4, "weighted", (3, 0, 1, 1)),
    ]:
        cases.append({"total": total, "world": world, "schedule": schedule, "weights": list(weights),
                      "indices": [list(work_indices(total, r, world, schedule, weights))
                                  for r in range(world)]})
    seeds = [{"base": b, "index": i, "seed": sample_seed(b, i)}
             for b in (0, 4, 12345, 2 ** 40 + 7) for i in (0, 1, 2, 3, 4, 199)]
    noise = []
    for base, idx in ((4, 0), (4, 3), (0, 1)):
        with torch.random.fork_rng(devices=[]):
            gen = torch.Generator(device="cpu").manual_seed(sample_seed(base, idx))
            torch.set_rng_state(gen.get_state())
            x = torch.randn(2, 3, 3) * 160.0
        noise.append({"base": base, "index": idx, "shape": [2, 3, 3], "scale": 160.0,
                      "values": x.flatten().tolist()})
    OUT.write_text(json.dumps({"work_indices": cases, "sample_seed": seeds, "noise": noise},
                              indent=1) + "\n")
    print(f"wrote {OUT}")


if __name__ == "__main__":
    main()
