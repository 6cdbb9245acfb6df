"""Diffusion samples over two GPUs (NCCL): rank 0's conditioning is broadcast,
each rank denoises its samples through the CUDA DiffusionTransformer, and every
rank ends with all samples, identical to one process running them all."""

import datetime
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from xfold_cpu_b200 import samples
from xfold_cpu_b200.nn import DiffusionTransformer, init_params_

pytestmark = pytest.mark.gpu

N, C, NUM_SAMPLES = 64, 768, 5


def _conditioning():
    g = torch.Generator().manual_seed(21)
    return {"single_cond": torch.randn(N, 384, generator=g),
            "pair_cond": torch.randn(N, N, 128, generator=g),
            "mask": (torch.arange(N) < N - 4).float()}


def _run(dev, emb):
    mod = DiffusionTransformer(c_act=C, num_blocks=2, super_block_size=2).eval()
    init_params_(mod, seed=11, std=0.05, perturb_layer_norm=True)
    mod = mod.to(dev)

    def denoise(x, i):
        a = x.clone()
        with torch.inference_mode():
            for _ in range(2):  # two denoising steps of the token transformer
                mod(a, emb["mask"], emb["single_cond"], emb["pair_cond"])
        return a

    return samples.sample_diffusion(denoise, (N, C), NUM_SAMPLES, 4, 1.0, dev)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, results):
    import torch.distributed as dist

    os.environ.update({"MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port),
                       "NCCL_NVLS_ENABLE": "0"})
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=120))
    try:
        emb = samples.broadcast_tensors(_conditioning() if rank == 0 else None, dev)
        results[rank] = _run(dev, emb).cpu()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_samples_over_two_gpus_match_one_process():
    dev = torch.device("cuda", 0)
    ref = _run(dev, {k: v.to(dev) for k, v in _conditioning().items()}).cpu()
    world = 2
    port = _free_port()
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    results = manager.dict()
    procs = [ctx.Process(target=_worker, args=(r, world, port, results)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=600)
        assert p.exitcode == 0
    assert torch.isfinite(ref).all()
    for r in range(world):
        assert torch.equal(results[r], ref)
