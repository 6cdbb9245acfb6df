"""Independent diffusion samples spread over GPUs (one process per GPU).

The reference's sample parallelism (xfold/alphafold3.py:489-505 and :397-439,
xfold/distributed.py) runs the trunk on rank 0, broadcasts its embeddings,
lets every rank denoise the samples its work schedule assigns it, each from a
noise draw seeded by the sample's index alone, and finally gives every rank
every sample.  This module does the same over torch.distributed (NCCL on GPUs,
gloo in the CPU tests):

  broadcast_tensors   rank 0's trunk outputs to every rank (once)
  work_indices        which samples a rank runs (cyclic / block / weighted,
                      the reference's schedules)
  sample_seed         the reference's per-sample seed, so a sample's initial
                      noise does not depend on the rank or the world size
  sample_diffusion    the local samples through a caller-supplied denoiser,
                      then every sample broadcast from the rank that owns it

The denoiser is the caller's (e.g. DiffusionTransformer steps or their CUDA
graph); samples are independent, so there is no collective inside it.
"""

from __future__ import annotations

import hashlib
from typing import Callable

import torch


def work_indices(total: int, rank: int, world_size: int, schedule: str = "cyclic",
                 weights: tuple[int, ...] = ()) -> range:
    """The samples rank `rank` of `world_size` runs: every index in [0, total)
    exactly once over all ranks, ranks without work allowed
    (xfold/distributed.py:14-37)."""
    if type(total) is not int or total < 0 or type(world_size) is not int or world_size < 1:
        raise ValueError("total must be a non-negative int and world_size a positive int")
    if type(rank) is not int or not 0 <= rank < world_size:
        raise ValueError("rank must lie in [0, world_size)")
    if schedule in ("cyclic", "block") and weights:
        raise ValueError("rank weights need the weighted schedule")
    if schedule == "cyclic":
        return range(rank, total, world_size)
    if schedule == "block":
        per, extra = divmod(total, world_size)
        start = rank * per + min(rank, extra)
        return range(start, start + per + (1 if rank < extra else 0))
    if schedule == "weighted":
        if (len(weights) != world_size or sum(weights) <= 0
                or any(type(w) is not int or w < 0 for w in weights)):
            raise ValueError("weighted schedule needs one non-negative int weight per rank, "
                             "summing to more than zero")
        wsum = sum(weights)
        return range(total * sum(weights[:rank]) // wsum, total * sum(weights[:rank + 1]) // wsum)
    raise ValueError("schedule must be 'cyclic', 'block' or 'weighted'")


def sample_seed(base_seed: int, sample_index: int) -> int:
    """Seed of sample `sample_index`'s noise: the first 8 bytes of
    BLAKE2b("xfold-sample-v1:<base>:<index>") as a big-endian integer, modulo
    2^63 (xfold/distributed.py:49-54).  Rank, world size and schedule do not
    enter it."""
    if type(sample_index) is not int or sample_index < 0:
        raise ValueError("sample_index must be a non-negative int")
    digest = hashlib.blake2b(f"xfold-sample-v1:{base_seed}:{sample_index}".encode("ascii"),
                             digest_size=8).digest()
    return int.from_bytes(digest, "big") % (2 ** 63)


def broadcast_tensors(tensors: dict[str, torch.Tensor] | None, device: torch.device,
                      group=None, src: int = 0) -> dict[str, torch.Tensor]:
    """Rank `src` passes its tensors (e.g. the trunk's pair / single
    embeddings); every rank returns them on `device`.  Names, shapes and dtypes
    travel first, then one broadcast per tensor in name order."""
    import torch.distributed as dist

    rank = dist.get_rank(group)
    meta = [None]
    if rank == src:
        if tensors is None:
            raise ValueError("the source rank must pass its tensors")
        meta[0] = [(k, tuple(v.shape), v.dtype) for k, v in sorted(tensors.items())]
    dist.broadcast_object_list(meta, src=src, group=group)
    out = {}
    for name, shape, dtype in meta[0]:
        if rank == src:
            t = tensors[name].to(device).contiguous()
        else:
            t = torch.empty(shape, dtype=dtype, device=device)
        dist.broadcast(t, src=src, group=group)
        out[name] = t
    return out


def sample_diffusion(denoise: Callable[[torch.Tensor, int], torch.Tensor],
                     shape: tuple[int, ...], num_samples: int, base_seed: int,
                     init_scale: float, device: torch.device, group=None,
                     schedule: str = "cyclic", weights: tuple[int, ...] = ()) -> torch.Tensor:
    """Runs this rank's samples and returns all `num_samples` of them on every
    rank, [num_samples, *shape] f32.

    Sample i starts from init_scale * N(0, 1) drawn on the CPU with a generator
    seeded by sample_seed(base_seed, i) (the reference draws the first noise
    level times a standard normal the same way, xfold/alphafold3.py:415-420),
    then `denoise(x, i)` returns its final state.  Without an initialised
    process group the call runs every sample in this process."""
    import torch.distributed as dist

    parallel = dist.is_available() and dist.is_initialized()
    world = dist.get_world_size(group) if parallel else 1
    rank = dist.get_rank(group) if parallel else 0
    out = torch.empty((num_samples, *shape), dtype=torch.float32, device=device)
    for i in work_indices(num_samples, rank, world, schedule, weights):
        g = torch.Generator(device="cpu").manual_seed(sample_seed(base_seed, i))
        x = (torch.randn(shape, generator=g) * init_scale).to(device)
        out[i] = denoise(x, i).to(torch.float32)
    if parallel:
        for src in range(world):
            global_src = dist.get_global_rank(group, src) if group is not None else src
            for i in work_indices(num_samples, src, world, schedule, weights):
                dist.broadcast(out[i], src=global_src, group=group)
    return out
