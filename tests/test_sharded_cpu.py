"""Row-sharded Pairformer block on the CPU: the exchange logic of
xfold_cpu_b200/sharded.py with the float32 restatement of each row-block stage
(oracle/stages.py), against the whole-pair oracle block.

Two exchanges are covered: all shards in one process (LocalExchange, G = 2 and
4) and one shard per process over gloo (ProcessGroupExchange, world_size 2 and
4).  A planted mistake in the exchange (chunks delivered in the wrong order)
must be caught."""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

import oracle
from oracle.stages import OracleStages
from xfold_cpu_b200 import sharded
from xfold_cpu_b200.nn import PairformerBlock, init_params_

N = 32
TOL = 1e-5


def _problem(seed=3):
    torch.manual_seed(seed)
    blk = PairformerBlock(c_pair=128, c_single=384).eval()
    init_params_(blk, seed=seed, std=0.05, perturb_layer_norm=True)
    pair = torch.randn(N, N, 128)
    single = torch.randn(N, 384)
    seq = torch.ones(N)
    seq[-5:] = 0
    pair_mask = seq[:, None] * seq[None, :]
    return blk, pair, single, seq, pair_mask


def _reference(blk, pair, single, seq, pair_mask):
    params = {k: v.float() for k, v in blk.state_dict().items()}
    with torch.no_grad():
        return oracle.pairformer_block(pair, pair_mask, single, seq, params)


def _run_local(exchange, blk, pair, single, seq, pair_mask):
    g = exchange.world
    pairs = [pair[sharded.shard_rows(N, g, r)].clone() for r in range(g)]
    s = single.clone()
    with torch.no_grad():
        sharded.pairformer_block(blk, pairs, pair_mask, s, seq, exchange, stages=OracleStages())
    return torch.cat(pairs), s


@pytest.mark.parametrize("world", [2, 4])
def test_local_exchange_matches_whole_pair(world):
    blk, pair, single, seq, pair_mask = _problem()
    ref_p, ref_s = _reference(blk, pair, single, seq, pair_mask)
    got_p, got_s = _run_local(sharded.LocalExchange(world), blk, pair, single, seq, pair_mask)
    assert (ref_p - pair).abs().max() > 1.0  # the block changes the pair
    assert oracle.relative_error(got_p - pair, ref_p - pair) <= TOL
    assert oracle.relative_error(got_s - single, ref_s - single) <= TOL


class _SwappedChunks(sharded.LocalExchange):
    """A wrong exchange: every all-to-all delivers its chunks in reverse order."""

    def all_to_all(self, bufs):
        return [t.flip(0) for t in super().all_to_all(bufs)]


def test_wrong_chunk_order_is_caught():
    blk, pair, single, seq, pair_mask = _problem()
    ref_p, _ = _reference(blk, pair, single, seq, pair_mask)
    got_p, _ = _run_local(_SwappedChunks(2), blk, pair, single, seq, pair_mask)
    assert oracle.relative_error(got_p - pair, ref_p - pair) > 0.1


def test_sharding_rejects_uneven_splits():
    with pytest.raises(ValueError, match="divisible"):
        sharded.check_sharding(30, 128, 4)
    with pytest.raises(ValueError, match="N % 8"):
        sharded.check_sharding(36, 128, 4)
    assert sharded.shard_rows(32, 4, 2) == slice(16, 24)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, results):
    import torch.distributed as dist

    os.environ.update({"MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port)})
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        blk, pair, single, seq, pair_mask = _problem()
        rows = sharded.shard_rows(N, world, rank)
        mine = [pair[rows].clone()]
        s = single.clone()
        with torch.no_grad():
            sharded.pairformer_block(blk, mine, pair_mask, s, seq,
                                     sharded.ProcessGroupExchange(), stages=OracleStages())
        gathered = [torch.empty_like(mine[0]) for _ in range(world)]
        dist.all_gather(gathered, mine[0])
        if rank == 0:
            ref_p, ref_s = _reference(blk, pair, single, seq, pair_mask)
            results["pair"] = oracle.relative_error(torch.cat(gathered) - pair, ref_p - pair)
        results[f"single{rank}"] = float(s.sum())
        if rank == 0:
            results["single_ref"] = float(_reference(blk, pair, single, seq, pair_mask)[1].sum())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_gloo_ranks_match_whole_pair(world):
    port = _free_port()
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()  # spawned, not forked: this process may hold a CUDA context
    results = manager.dict()
    procs = [ctx.Process(target=_worker, args=(r, world, port, results)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        assert p.exitcode == 0
    assert results["pair"] <= TOL
    singles = [results[f"single{r}"] for r in range(world)]
    assert all(v == singles[0] for v in singles)  # every rank's single copy agrees
    assert abs(singles[0] - results["single_ref"]) <= 1e-3 * max(1.0, abs(results["single_ref"]))
