"""Diffusion samples spread over ranks (xfold_cpu_b200/samples.py) on CPU.

The work schedule, the per-sample seed and the initial noise are pinned by
tests/golden/distributed.json, made by running the reference's own
xfold/distributed.py (tests/golden/make_distributed_golden.py).  gloo ranks
(world size 2 and 3) must produce exactly the samples of one process."""

import json
import os
import socket
from pathlib import Path

import pytest
import torch
import torch.multiprocessing as mp

from xfold_cpu_b200 import samples

GOLDEN = json.loads((Path(__file__).resolve().parent / "golden" / "distributed.json").read_text())


def test_work_indices_match_reference():
    for case in GOLDEN["work_indices"]:
        got = [list(samples.work_indices(case["total"], r, case["world"], case["schedule"],
                                         tuple(case["weights"])))
               for r in range(case["world"])]
        assert got == case["indices"], case
        flat = sorted(i for idx in got for i in idx)
        assert flat == list(range(case["total"]))  # disjoint, complete


@pytest.mark.parametrize("args", [(5, 2, 2, "cyclic", ()), (5, -1, 2, "cyclic", ()),
                                  (5, 0, 2, "cyclic", (1, 1)), (5, 0, 2, "spiral", ()),
                                  (5, 0, 2, "weighted", (0, 0)), (-1, 0, 1, "cyclic", ())])
def test_work_indices_reject_bad_arguments(args):
    with pytest.raises(ValueError):
        samples.work_indices(*args)


def test_sample_seed_matches_reference():
    for case in GOLDEN["sample_seed"]:
        assert samples.sample_seed(case["base"], case["index"]) == case["seed"]
    with pytest.raises(ValueError):
        samples.sample_seed(0, -1)


def test_initial_noise_matches_reference():
    for case in GOLDEN["noise"]:
        out = samples.sample_diffusion(lambda x, i: x, tuple(case["shape"]), case["index"] + 1,
                                       case["base"], case["scale"], torch.device("cpu"))
        assert torch.equal(out[case["index"]].flatten(), torch.tensor(case["values"]))


def _denoise_with(emb):
    # stands in for the denoising steps: depends on the broadcast embedding,
    # the sample's own noise and its index
    def denoise(x, i):
        for _ in range(3):
            x = torch.tanh(x * 0.01 + emb["pair"].mean(dim=(0, 1))[: x.shape[-1]]) + 0.1 * i
        return x
    return denoise


def _embeddings():
    g = torch.Generator().manual_seed(7)
    return {"pair": torch.randn(6, 6, 4, generator=g), "single": torch.randn(6, 8, generator=g)}


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, schedule, results):
    import torch.distributed as dist

    os.environ.update({"MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port)})
    dist.init_process_group("gloo", rank=rank, world_size=world)
    cpu = torch.device("cpu")
    emb = samples.broadcast_tensors(_embeddings() if rank == 0 else None, cpu)
    out = samples.sample_diffusion(_denoise_with(emb), (5, 3), 5, 4, 160.0, cpu,
                                   schedule=schedule)
    results[rank] = (out.tolist(), {k: v.tolist() for k, v in emb.items()})
    dist.destroy_process_group()


@pytest.mark.parametrize("world,schedule", [(2, "cyclic"), (3, "block")])
def test_gloo_ranks_match_one_process(world, schedule):
    cpu = torch.device("cpu")
    ref = samples.sample_diffusion(_denoise_with(_embeddings()), (5, 3), 5, 4, 160.0, cpu)
    port = _free_port()
    manager = mp.Manager()
    results = manager.dict()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_worker, args=(r, world, port, schedule, results))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    emb = {k: v.tolist() for k, v in _embeddings().items()}
    for r in range(world):
        out, got_emb = results[r]
        assert got_emb == emb
        assert torch.equal(torch.tensor(out), ref)
