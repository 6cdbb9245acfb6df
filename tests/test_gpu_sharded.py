"""Row-block stages and the row-sharded Pairformer block on the GPU.

The stage entry points (xfb_triangle_projection / _output,
xfb_grid_attention_prepare / _rows, xfb_pair_logits_rows, with xfb_gemm for
the channel-shard contraction) are checked one by one against the float32
restatement of the same stages (oracle/stages.py).  The sharded block is then
checked end to end against the whole-pair oracle block: all shards on one GPU
(LocalExchange, G = 2 and 4), and, when the box has two GPUs, one shard per
GPU over NCCL."""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

import oracle
from oracle.stages import OracleStages
from xfold_cpu_b200 import _capi, native, sharded
from xfold_cpu_b200.nn import GridSelfAttention, PairformerBlock, TriangleMultiplication, init_params_

pytestmark = pytest.mark.gpu

TOL = 1e-2
DEV = torch.device("cuda")
LOG2E = 1.4426950408889634


@pytest.fixture(autouse=True)
def _no_device_error():
    _capi.device_error(clear=True)
    yield
    torch.cuda.synchronize()
    assert _capi.device_error(clear=True) == 0


def _masks(n, tail):
    seq = torch.ones(n)
    seq[-tail:] = 0
    return seq, seq[:, None] * seq[None, :]


def _rel(got, ref):
    return oracle.relative_error(got.float().cpu(), ref.float())


@pytest.mark.parametrize("outgoing", [True, False])
def test_triangle_stages_match_restatement(outgoing):
    rows, n = 40, 96
    mod = TriangleMultiplication(128, _outgoing=outgoing).eval()
    init_params_(mod, seed=11, perturb_layer_norm=True)
    g = torch.Generator().manual_seed(12)
    pair = torch.randn(rows, n, 128, generator=g)
    _, pmask = _masks(n, 7)
    mask_rows = pmask[:rows]
    ora = OracleStages()
    with torch.no_grad():
        a_ref, b_ref, g_ref = ora.trimul_project(mod, pair, mask_rows)
    dmod = mod.to(DEV)
    with torch.inference_mode():
        a, b, gate = sharded.NativeStages().trimul_project(dmod, pair.to(DEV), mask_rows.to(DEV))
        assert a.shape == (128, rows, n) and gate.shape == (rows, n, 128)
        assert _rel(a, a_ref) < TOL and _rel(b, b_ref) < TOL and _rel(gate, g_ref) < TOL
        # contraction of a channel shard over a square block, then the output stage
        sq_a = torch.randn(16, n, n, generator=g)
        sq_b = torch.randn(16, n, n, generator=g)
        z = native.triangle_contraction(sq_a.to(DEV), sq_b.to(DEV), outgoing)
        z_ref = ora.trimul_contract(dmod, sq_a, sq_b)
        assert _rel(z, z_ref) < TOL
        z_rows = torch.randn(128, rows, n, generator=g)
        out = torch.zeros(rows, n, 128, device=DEV)
        sharded.NativeStages().trimul_output(dmod, z_rows.to(DEV), g_ref.to(DEV), out)
    ref = torch.zeros(rows, n, 128)
    with torch.no_grad():
        ora.trimul_output(mod.cpu(), z_rows, g_ref, ref)
    assert _rel(out, ref) < TOL


@pytest.mark.parametrize("rows,n", [(32, 64), (24, 104)])
def test_attention_stages_match_restatement(rows, n):
    mod = GridSelfAttention(128, 4).eval()
    init_params_(mod, seed=13, std=0.05, perturb_layer_norm=True)
    g = torch.Generator().manual_seed(14)
    pair = torch.randn(rows, n, 128, generator=g)
    full_bias = torch.randn(4, n, n, generator=g)
    _, pmask = _masks(n, 9)
    ora = OracleStages()
    with torch.no_grad():
        x_ref, bias_ref = ora.attention_prepare(mod, pair)
        upd_ref = ora.attention_rows(mod, x_ref, pmask[:rows], full_bias)
    dmod = mod.to(DEV)
    with torch.inference_mode():
        x, bias = sharded.NativeStages().attention_prepare(dmod, pair.to(DEV))
        scale = LOG2E if n % 8 == 0 else 1.0  # stage-1 bias units (head dim 32)
        assert bias.shape == (4, rows, n)
        assert _rel(x, x_ref) < TOL and _rel(bias.float() / scale, bias_ref) < TOL
        upd = sharded.NativeStages().attention_rows(dmod, x_ref.to(DEV), pmask[:rows].to(DEV),
                                                    (full_bias * scale).to(DEV))
    assert _rel(upd, upd_ref) < TOL


def test_pair_logits_rows():
    rows, n = 16, 72
    block = PairformerBlock().eval()
    init_params_(block, seed=15, perturb_layer_norm=True)
    pair = torch.randn(rows, n, 128, generator=torch.Generator().manual_seed(16))
    with torch.no_grad():
        ref = OracleStages().pair_logits_rows(block, pair)
    block = block.to(DEV)
    with torch.inference_mode():
        got = sharded.NativeStages().pair_logits_rows(block, pair.to(DEV))
    assert got.shape == (16, rows, n) and _rel(got, ref) < TOL


def _problem(n, seed=17):
    block = PairformerBlock().eval()
    init_params_(block, seed=seed, perturb_layer_norm=True)
    g = torch.Generator().manual_seed(seed + 1)
    pair = torch.randn(n, n, 128, generator=g)
    single = torch.randn(n, 384, generator=g)
    seq, pmask = _masks(n, 5)
    return block, pair, single, seq, pmask


@pytest.mark.parametrize("routed", [False, True])
@pytest.mark.parametrize("world,n", [(2, 64), (4, 128)])
def test_sharded_block_on_one_gpu(world, n, routed):
    block, pair, single, seq, pmask = _problem(n)
    params = {k: v.detach().clone() for k, v in block.state_dict().items()}
    ref_p, ref_s = oracle.pairformer_block(pair, pmask, single, seq, params)
    block = block.to(DEV)
    pairs = [pair[sharded.shard_rows(n, world, r)].to(DEV).contiguous() for r in range(world)]
    s = single.to(DEV)
    with torch.inference_mode():
        sharded.pairformer_block(block, pairs, pmask.to(DEV), s, seq.to(DEV),
                                 sharded.LocalExchange(world, routed=routed))
        whole_p, whole_s = pair.to(DEV), single.to(DEV)
        block(whole_p, pmask.to(DEV), whole_s, seq.to(DEV))
    got = torch.cat([p.cpu() for p in pairs])
    assert oracle.relative_error(got - pair, ref_p - pair) < TOL
    assert oracle.relative_error(s.cpu() - single, ref_s - single) < TOL
    # and close to the single-GPU block (same kernels, different blocking)
    assert oracle.relative_error(got - pair, whole_p.cpu() - pair) < TOL


@pytest.mark.parametrize("world,n", [(2, 96), (4, 128), (8, 256)])
def test_routed_stages_match_copy_exchange(world, n):
    """The routed stages store exactly what the copy exchanges move: two
    blocks, shards on one GPU, bit-identical pair and single."""
    block, pair, single, seq, pmask = _problem(n, seed=29)
    block = block.to(DEV)
    out = {}
    for routed in (False, True):
        pairs = [pair[sharded.shard_rows(n, world, r)].to(DEV).contiguous()
                 for r in range(world)]
        s = single.to(DEV)
        ex = sharded.LocalExchange(world, routed=routed)
        with torch.inference_mode():
            for _ in range(2):
                sharded.pairformer_block(block, pairs, pmask.to(DEV), s, seq.to(DEV), ex)
        out[routed] = (torch.cat(pairs).cpu(), s.cpu())
    assert torch.equal(out[True][0], out[False][0])
    assert torch.equal(out[True][1], out[False][1])


def test_self_attention_rows_match_whole_track():
    """Query-row shards of the single attention put together equal the whole
    track's update (same kernels on the same tokens)."""
    n, world = 256, 4
    block, pair, single, seq, pmask = _problem(n, seed=31)
    block = block.to(DEV)
    st = sharded.NativeStages()
    with torch.inference_mode():
        p = pair.to(DEV)
        logits = native.pair_logits(p, block.single_pair_logits_norm.weight,
                                    block.single_pair_logits_norm.bias,
                                    block.single_pair_logits_norm.eps,
                                    block.single_pair_logits_projection.weight)
        whole = single.to(DEV)
        block.single_attention_.accumulate_(whole, seq.to(DEV), logits)
        x_in = single.to(DEV)
        parts = x_in.clone()
        rows = n // world
        for r in range(world):
            st.single_attention_rows(block, x_in, seq.to(DEV),
                                     logits[:, r * rows:(r + 1) * rows].contiguous(),
                                     r * rows, parts)
    assert _rel(parts - single.to(DEV), (whole - single.to(DEV)).cpu()) < 1e-3


def _free_port():
    with socket.socket() as sock:
        sock.bind(("127.0.0.1", 0))
        return sock.getsockname()[1]


def _nccl_worker(rank, world, port, n, results):
    import datetime

    import torch.distributed as dist

    os.environ.update({"MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port),
                       "NCCL_NVLS_ENABLE": "0"})
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=120))
    try:
        block, pair, single, seq, pmask = _problem(n)
        params = {k: v.detach().clone() for k, v in block.state_dict().items()}
        block = block.to(dev)
        mine = [pair[sharded.shard_rows(n, world, rank)].to(dev).contiguous()]
        s = single.to(dev)
        with torch.inference_mode():
            sharded.pairformer_block(block, mine, pmask.to(dev), s, seq.to(dev),
                                     sharded.ProcessGroupExchange())
            gathered = [torch.empty_like(mine[0]) for _ in range(world)]
            dist.all_gather(gathered, mine[0])
        torch.cuda.synchronize(dev)
        results[f"err{rank}"] = int(_capi.device_error(clear=True))
        if rank == 0:
            ref_p, ref_s = oracle.pairformer_block(pair, pmask, single, seq, params)
            got = torch.cat([t.cpu() for t in gathered])
            results["pair"] = oracle.relative_error(got - pair, ref_p - pair)
            results["single"] = oracle.relative_error(s.cpu() - single, ref_s - single)
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_sharded_block_over_nccl():
    world, n = 2, 128
    port = _free_port()
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()  # spawned, not forked: this process may hold a CUDA context
    results = manager.dict()
    procs = [ctx.Process(target=_nccl_worker, args=(r, world, port, n, results))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=600)
        assert p.exitcode == 0
    assert results["err0"] == 0 and results["err1"] == 0
    assert results["pair"] < TOL and results["single"] < TOL


def _peer_worker(rank, world, port, n, results):
    import datetime

    import torch.distributed as dist

    os.environ.update({"MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port),
                       "NCCL_NVLS_ENABLE": "0"})
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=120))
    try:
        peer, coll = sharded.PeerExchange(), sharded.ProcessGroupExchange()
        g = torch.Generator(device=dev).manual_seed(100 + rank)
        rows = n // world
        cases = {
            "rows_to_channels": torch.randn(128, rows, n, device=dev, generator=g).bfloat16(),
            "channels_to_rows": torch.randn(128 // world, n, n, device=dev, generator=g).bfloat16(),
            "gather_rows": torch.randn(4, rows, n, device=dev, generator=g).bfloat16(),
            "transpose": torch.randn(rows, n, 128, device=dev, generator=g).bfloat16(),
        }
        same = {}
        for name, t in cases.items():
            for _ in range(3):  # both receive copies and a reuse of the first
                got = getattr(peer, name)([t])[0].clone()
                want = getattr(coll, name)([t])[0]
                same[name] = bool(torch.equal(got, want))
                if not same[name]:
                    break
        results[f"same{rank}"] = same
        block, pair, single, seq, pmask = _problem(n)
        params = {k: v.detach().clone() for k, v in block.state_dict().items()}
        block = block.to(dev)
        mine = [pair[sharded.shard_rows(n, world, rank)].to(dev).contiguous()]
        s = single.to(dev)
        copied = [mine[0].clone()]
        s_copied = s.clone()
        unrouted = sharded.PeerExchange(routed=False)
        with torch.inference_mode():
            for _ in range(2):  # two blocks: the exchanges reuse their receive buffers
                sharded.pairformer_block(block, mine, pmask.to(dev), s, seq.to(dev), peer)
            for _ in range(2):  # the same blocks with copy exchanges instead of routed stages
                sharded.pairformer_block(block, copied, pmask.to(dev), s_copied, seq.to(dev),
                                         unrouted)
            results[f"routed_same{rank}"] = bool(torch.equal(mine[0], copied[0]) and
                                                 torch.equal(s, s_copied))
            # one block captured into a CUDA graph (device-side barrier epochs),
            # replayed twice: the same two blocks again
            g_pair = [pair[sharded.shard_rows(n, world, rank)].to(dev).contiguous()]
            g_single = single.to(dev)
            g_pm, g_seq = pmask.to(dev), seq.to(dev)
            torch.cuda.synchronize(dev)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                sharded.pairformer_block(block, g_pair, g_pm, g_single, g_seq, peer)
            for _ in range(2):
                graph.replay()
            torch.cuda.synchronize(dev)
            results[f"graph_same{rank}"] = bool(torch.equal(g_pair[0], mine[0]) and
                                                torch.equal(g_single, s))
            del graph
            # the single track on its own stream and exchange, overlapping the
            # next block's pair operators: the same two blocks
            side, side_ex = torch.cuda.Stream(dev), sharded.PeerExchange()
            o_pair = [pair[sharded.shard_rows(n, world, rank)].to(dev).contiguous()]
            o_single = single.to(dev)
            for _ in range(2):
                sharded.pairformer_block(block, o_pair, g_pm, o_single, g_seq, peer,
                                         single_stream=side, single_exchange=side_ex)
            torch.cuda.current_stream(dev).wait_stream(side)
            torch.cuda.synchronize(dev)
            results[f"overlap_same{rank}"] = bool(torch.equal(o_pair[0], mine[0]) and
                                                  torch.equal(o_single, s))
            gathered = [torch.empty_like(mine[0]) for _ in range(world)]
            dist.all_gather(gathered, mine[0])
        torch.cuda.synchronize(dev)
        results[f"err{rank}"] = int(_capi.device_error(clear=True))
        if rank == 0:
            ref_p, ref_s = oracle.pairformer_block(pair, pmask, single, seq, params)
            ref_p, ref_s = oracle.pairformer_block(ref_p, pmask, ref_s, seq, params)
            got = torch.cat([t.cpu() for t in gathered])
            results["pair"] = oracle.relative_error(got - pair, ref_p - pair)
            results["single"] = oracle.relative_error(s.cpu() - single, ref_s - single)
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_peer_exchange_over_nvlink():
    world, n = 2, 128
    port = _free_port()
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    results = manager.dict()
    procs = [ctx.Process(target=_peer_worker, args=(r, world, port, n, results))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=600)
        assert p.exitcode == 0
    for r in range(world):
        assert all(results[f"same{r}"].values()), results[f"same{r}"]
        assert results[f"routed_same{r}"]
        assert results[f"graph_same{r}"]
        assert results[f"overlap_same{r}"]
        assert results[f"err{r}"] == 0
    assert results["pair"] < TOL and results["single"] < TOL
