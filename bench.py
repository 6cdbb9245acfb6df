"""Benchmark: Pairformer block time at N_token = 1024, bf16, on B200.

Workload: a 48-block Pairformer trunk, N_token = 1024,
c_pair = 128, c_single = 384, random-init weights ~N(0, 0.02) (LayerNorm
gamma = 1, beta = 0), pair and single ~N(0, 1), pair mask = outer product of a
sequence mask with a padded tail of 64 tokens, seed 3.  One step = one pass of
the trunk (48 blocks); the metric is ms per block = step time / 48.

  value  device-resident: pair / single already in HBM, CUDA events around
         exactly K steps on the launching stream (max over ranks).
  e2e    the same metric through the public module API with host buffers:
         every step copies pair / single / masks from pinned host memory and
         reads pair / single back, inside the timed region.
  roofline  the dominant kernels timed live with CUDA events (same shapes as
         inside the block): the triangle-attention flash kernel and the
         triangle contraction GEMM, FLOPs / time against the measured bf16 peak.
  cpu_baseline  the reference's own PairformerBlock (baseline/_ref, torch
         backend, CPU bf16 autocast) on this host's cores, one C4 block at
         N = 1024, each of its seven sub-modules timed once (the CPU oracle
         under the same autocast when the reference is not installed).
  parity / parity_fp32  checkers after the timed regions: block 0 at N = 1024
         against the CPU oracle (bf16 bar 1e-2), and BASELINE C1 (N = 256,
         float32 path) against the reference's own block in float32 (1e-4).

`--impl reference` times that CPU path alone on the same metric (the reference
arm); under torchrun only rank 0 runs it.

Multi-GPU (--gpus N under torchrun): one N = 1024 trunk with its pair
row-sharded over the N GPUs (rank r holds rows [rN/G, (r+1)N/G)); the routed
stages store each exchanged tensor straight into the peers' receive buffers
over NVLink, the single track runs on its own stream, and the trunk is
replayed as one CUDA graph ("scaling": "strong"); value = the per-block time
of the slowest rank.
"""

from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "Pairformer block ms at N_tok=1024 bf16"
UNIT = "ms/block"
N_TOKEN = 1024
N_BLOCKS = 48
C_PAIR, C_SINGLE = 128, 384
SEED = 3


def _peaks() -> dict:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return {"hbm_gbs": data["hbm_gbs"], "bf16_tflops": data["bf16_tflops"],
                "bf16_tflops_sustained": data.get("bf16_tflops_sustained"), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
            "source": "fallback"}


def _inputs(n: int, seed: int):
    import torch

    g = torch.Generator().manual_seed(seed)
    pair = torch.randn(n, n, C_PAIR, generator=g)
    single = torch.randn(n, C_SINGLE, generator=g)
    seq_mask = torch.ones(n)
    seq_mask[-64:] = 0
    pair_mask = seq_mask[:, None] * seq_mask[None, :]
    return pair, pair_mask, single, seq_mask


class ClockSampler:
    """nvidia-smi clock / throttle sampling during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.device_index = device_index
        self.proc = None
        self.path = Path(os.environ.get("TMPDIR", "/tmp")) / f"xfb_clocks_{os.getpid()}.csv"

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.device_index}", f"--query-gpu={self.QUERY}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        for line in self.path.read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                rows.append(parts)
        self.path.unlink(missing_ok=True)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = sorted(float(r[1]) for r in rows if r[1].replace(".", "").isdigit())
        smax = max((float(r[2]) for r in rows if r[2].replace(".", "").isdigit()), default=None)
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": sm[len(sm) // 2] if sm else None, "sm_max_mhz": smax,
                "reasons": reasons, "samples": len(rows)}


def _dist():
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1 and not dist.is_initialized():
        import datetime

        backend = "nccl" if torch.cuda.is_available() else "gloo"
        if backend == "nccl":
            torch.cuda.set_device(local)
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=300))
    return world, rank, local


def _max_over_ranks(value: float, world: int) -> float:
    if world == 1:
        return value
    import torch
    import torch.distributed as dist

    t = torch.tensor([value], dtype=torch.float64,
                     device="cuda" if dist.get_backend() == "nccl" else "cpu")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _barrier(world: int):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


# ----------------------------------------------------------------------------- CPU baseline

REF_DIR = ROOT / "baseline" / "_ref"
# The seven sub-modules of one Pairformer block, in the order of
# xfold/nn/pairformer.py:96-112; one reference step runs one of them.
BLOCK_PARTS = ("triangle_multiplication_outgoing", "triangle_multiplication_incoming",
               "pair_attention1", "pair_attention2", "pair_transition", "single_attention",
               "single_transition")


def _host_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:  # pragma: no cover
        return os.cpu_count() or 1


def _reference_parts(n: int):
    """The block's seven sub-module calls on the reference's CPU path, with
    the C4 weights (block 0: init seed 3000) and inputs (seed 3).

    Preferred: the reference's own torch modules (xfold.nn.pairformer
    PairformerBlock, installed unmodified in baseline/_ref) under CPU bf16
    autocast, as its ModelRunner runs them (run_alphafold.py:466-472); the
    weights are copied in with load_state_dict (same parameter names).  If
    baseline/_ref is absent: the CPU oracle (a restatement of the same torch
    path) under the same autocast.  Returns (kind, callables, inputs)."""
    import torch

    from xfold_cpu_b200.nn import PairformerBlock, init_params_

    ours = PairformerBlock(c_pair=C_PAIR, c_single=C_SINGLE)
    init_params_(ours, seed=SEED * 1000)
    pair, pair_mask, single, seq_mask = _inputs(n, SEED)
    if (REF_DIR / "xfold").is_dir():
        if str(REF_DIR) not in sys.path:
            sys.path.insert(0, str(REF_DIR))
        from xfold.nn.pairformer import PairformerBlock as RefBlock

        ref = RefBlock(c_pair=C_PAIR, c_single=C_SINGLE).eval()
        ref.load_state_dict(ours.state_dict(), strict=True)

        def single_attention():
            logits = ref.single_pair_logits_projection(ref.single_pair_logits_norm(pair))
            single.add_(ref.single_attention_(single, seq_mask, pair_logits=logits.permute(2, 0, 1)))

        parts = {
            "triangle_multiplication_outgoing":
                lambda: pair.add_(ref.triangle_multiplication_outgoing(pair, mask=pair_mask)),
            "triangle_multiplication_incoming":
                lambda: pair.add_(ref.triangle_multiplication_incoming(pair, mask=pair_mask)),
            "pair_attention1": lambda: pair.add_(ref.pair_attention1(pair, mask=pair_mask)),
            "pair_attention2": lambda: pair.add_(ref.pair_attention2(pair, mask=pair_mask)),
            "pair_transition": lambda: pair.add_(ref.pair_transition(pair)),
            "single_attention": single_attention,
            "single_transition": lambda: single.add_(ref.single_transition(single)),
        }
        return "reference", parts
    import oracle

    params = {k: v.detach().clone() for k, v in ours.state_dict().items()}
    parts = {
        "triangle_multiplication_outgoing": lambda: pair.add_(oracle.triangle_multiplication(
            pair, pair_mask, params, True, "triangle_multiplication_outgoing.")),
        "triangle_multiplication_incoming": lambda: pair.add_(oracle.triangle_multiplication(
            pair, pair_mask, params, False, "triangle_multiplication_incoming.")),
        "pair_attention1": lambda: pair.add_(oracle.grid_self_attention(
            pair, pair_mask, params, False, 4, "pair_attention1.")),
        "pair_attention2": lambda: pair.add_(oracle.grid_self_attention(
            pair, pair_mask, params, True, 4, "pair_attention2.")),
        "pair_transition": lambda: pair.add_(oracle.transition(pair, params, "pair_transition.")),
        "single_attention": lambda: single.add_(oracle.self_attention(
            single, seq_mask, oracle.pair_logits(pair, params), params, None, 16, False,
            "single_attention_.")),
        "single_transition": lambda: single.add_(oracle.transition(single, params,
                                                                   "single_transition.")),
    }
    return "port", parts


def _time_parts(parts: dict, order: list[str]) -> dict:
    """Runs the named sub-modules in order under CPU bf16 autocast; returns
    {name: [seconds, ...]}."""
    import torch

    times: dict[str, list[float]] = {}
    with torch.inference_mode(), torch.amp.autocast("cpu", dtype=torch.bfloat16):
        for name in order:
            t0 = time.perf_counter()
            parts[name]()
            times.setdefault(name, []).append(time.perf_counter() - t0)
    return times


def cpu_baseline(threads: int | None = None) -> dict:
    """One Pairformer block at N = 1024 (C4, bf16 autocast) on the reference's
    CPU path, timed sub-module by sub-module on this host's cores (about
    10-30 s of CPU work): ms per block = the sum of the seven calls."""
    import torch

    torch.set_num_threads(threads or _host_threads())
    kind, parts = _reference_parts(N_TOKEN)
    times = _time_parts(parts, list(BLOCK_PARTS))
    per = {k: round(v[0] * 1e3, 1) for k, v in times.items()}
    total = sum(v[0] for v in times.values())
    who = ("the reference's own torch modules (xfold.nn.pairformer, baseline/_ref)"
           if kind == "reference" else "the CPU oracle (restated reference torch path)")
    return {"value": round(total * 1e3, 1), "unit": UNIT, "cores": torch.get_num_threads(),
            "kind": kind, "per_part_ms": per,
            "sample": (f"1 Pairformer block at N={N_TOKEN} (C4 weights and inputs) under CPU bf16 "
                       f"autocast, {who}, its 7 sub-modules timed once each ({total:.1f} s); "
                       f"measured, not extrapolated")}


PARITY_TOL = 1e-2


def block_parity(dev, blk) -> dict:
    """Sampled-row parity of one C4 block at N = 1024 against the CPU oracle:
    each pair update (both triangle multiplications, both triangle attentions,
    the transition) is compared on seven sampled rows with the oracle applied
    to the same input, the single track in full; max |got - ref| / max |ref|
    per update (the bf16 bar is 1e-2).  Checker only: runs after the timed
    regions."""
    import torch

    import oracle

    n = N_TOKEN
    pair_h, pair_mask_h, single_h, seq_h = _inputs(n, SEED)
    params = {k: v.detach().float().cpu() for k, v in blk.state_dict().items()}
    rows = sorted({0, 1, n // 3, n // 2 + 7, n - 65, n - 64, n - 1})
    pair, pair_mask = pair_h.to(dev), pair_mask_h.to(dev)
    single, seq_mask = single_h.to(dev), seq_h.to(dev)
    err = {}
    ref_bf16 = None
    if (REF_DIR / "xfold").is_dir():
        # the reference's own bf16 autocast path on the same first input, for scale
        if str(REF_DIR) not in sys.path:
            sys.path.insert(0, str(REF_DIR))
        from xfold.nn.pairformer import PairformerBlock as RefBlock
        ref_blk = RefBlock(c_pair=C_PAIR, c_single=C_SINGLE).eval()
        ref_blk.load_state_dict({k: v.float().cpu() for k, v in blk.state_dict().items()},
                                strict=True)
        with torch.inference_mode():
            want = oracle.triangle_multiplication_rows(pair_h, pair_mask_h, params, True, rows,
                                                       "triangle_multiplication_outgoing.")
            with torch.amp.autocast("cpu", dtype=torch.bfloat16):
                got_ref = ref_blk.triangle_multiplication_outgoing(pair_h, mask=pair_mask_h)
            ref_bf16 = {"triangle_multiplication_outgoing":
                        round(oracle.relative_error(got_ref[rows].float(), want), 5)}
        del ref_blk, got_ref
    with torch.inference_mode():
        for name, transpose, ref_fn in (
            ("triangle_multiplication_outgoing", False, lambda x: oracle.triangle_multiplication_rows(
                x, pair_mask_h, params, True, rows, "triangle_multiplication_outgoing.")),
            ("triangle_multiplication_incoming", False, lambda x: oracle.triangle_multiplication_rows(
                x, pair_mask_h, params, False, rows, "triangle_multiplication_incoming.")),
            ("pair_attention1", False, lambda x: oracle.grid_self_attention_rows(
                x, pair_mask_h, params, False, rows, 4, "pair_attention1.")),
            ("pair_attention2", True, lambda x: oracle.grid_self_attention_rows(
                x, pair_mask_h, params, True, rows, 4, "pair_attention2.")),
            ("pair_transition", False, lambda x: oracle.transition(x[rows], params,
                                                                   "pair_transition.")),
        ):
            before = pair.clone()
            mod = getattr(blk, name)
            if name == "pair_transition":
                mod.accumulate_(pair)
            else:
                mod.accumulate_(pair, pair_mask)
            upd = pair - before
            got = (upd[:, rows].permute(1, 0, 2) if transpose else upd[rows]).float().cpu()
            del upd
            err[name] = oracle.relative_error(got, ref_fn(before.cpu()))
            del before
        norm = blk.single_pair_logits_norm
        from xfold_cpu_b200 import native

        logits = native.pair_logits(pair, norm.weight, norm.bias, norm.eps,
                                     blk.single_pair_logits_projection.weight.bfloat16())
        s0 = single.clone()
        blk.single_attention_.accumulate_(single, seq_mask, logits)
        ref_logits = oracle.pair_logits(pair.cpu(), params)
        err["single_attention"] = oracle.relative_error(
            (single - s0).cpu(), oracle.self_attention(s0.cpu(), seq_h, ref_logits, params, None,
                                                       16, False, "single_attention_."))
        s1 = single.clone()
        blk.single_transition.accumulate_(single)
        err["single_transition"] = oracle.relative_error(
            (single - s1).cpu(), oracle.transition(s1.cpu(), params, "single_transition."))
    worst = max(err.values())
    return {"max_rel_err": round(worst, 5), "tolerance": PARITY_TOL, "ok": worst <= PARITY_TOL,
            "per_update": {k: round(v, 5) for k, v in err.items()}, "rows": rows,
            "reference_bf16_per_update": ref_bf16,
            "what": "block 0 at N=1024 (C4), each update vs the CPU oracle on the same input, "
                    "sampled pair rows, single track in full"}


def fp32_parity(dev) -> dict:
    """BASELINE config C1 in float32: one Pairformer block at N = 256, seed 0,
    masks all ones, random init N(0, 0.02), run with the library's float32
    path (fastnn.config.compute_dtype = "float32") and with the reference's own
    PairformerBlock on the CPU in float32 (baseline/_ref; the CPU oracle when
    the reference is not installed); max |got - ref| / max |ref| of the pair
    and single updates (the north_star's fp32 bar is 1e-4).  Checker only: runs
    after the timed regions."""
    import torch

    from xfold_cpu_b200.fastnn import config
    from xfold_cpu_b200.nn import PairformerBlock, init_params_

    n = 256
    blk = PairformerBlock(c_pair=C_PAIR, c_single=C_SINGLE).eval()
    init_params_(blk, seed=0)
    g = torch.Generator().manual_seed(0)
    pair = torch.randn(n, n, C_PAIR, generator=g)
    single = torch.randn(n, C_SINGLE, generator=g)
    seq_mask = torch.ones(n)
    pair_mask = torch.ones(n, n)
    state = {k: v.detach().float().cpu().clone() for k, v in blk.state_dict().items()}
    with torch.inference_mode():
        if (REF_DIR / "xfold").is_dir():
            if str(REF_DIR) not in sys.path:
                sys.path.insert(0, str(REF_DIR))
            from xfold.nn.pairformer import PairformerBlock as RefBlock

            ref_blk = RefBlock(c_pair=C_PAIR, c_single=C_SINGLE).eval()
            ref_blk.load_state_dict(state, strict=True)
            ref_p, ref_s = ref_blk(pair.clone(), pair_mask, single.clone(), seq_mask)
            against = "the reference's PairformerBlock (torch backend, CPU float32)"
        else:
            import oracle

            ref_p, ref_s = oracle.pairformer_block(pair, pair_mask, single, seq_mask, state)
            against = "the CPU float32 oracle (baseline/_ref not installed)"
        old = config.compute_dtype
        config.compute_dtype = config.FLOAT32
        try:
            blk = blk.to(dev)
            p, s = pair.to(dev), single.to(dev)
            blk(p, pair_mask.to(dev), s, seq_mask.to(dev))
            torch.cuda.synchronize(dev)
        finally:
            config.compute_dtype = old
        import oracle

        pair_err = oracle.relative_error(p.cpu() - pair, ref_p - pair)
        single_err = oracle.relative_error(s.cpu() - single, ref_s - single)
    return {"pair_update_rel_err": float(f"{pair_err:.3g}"),
            "single_update_rel_err": float(f"{single_err:.3g}"), "tolerance": 1e-4,
            "ok": max(pair_err, single_err) <= 1e-4,
            "what": f"BASELINE C1 (one block, N=256, fp32, seed 0) with compute_dtype float32 "
                    f"vs {against}"}


def run_reference(args) -> None:
    """The reference arm: the reference's CPU path on C4's workload.  One step
    is one of the block's seven sub-modules at full size (N = 1024), taken in
    rotation, so a run of K steps covers K / 7 blocks; the value (ms per block)
    is the sum over the seven sub-modules of each one's mean time over the
    timed steps, plus the warm-up steps for any sub-module the timed steps did
    not reach (K < 7)."""
    world, rank, _ = _dist()
    if rank != 0:
        return
    import torch

    threads = _host_threads()
    torch.set_num_threads(threads)
    n = args.n  # N_TOKEN unless a smaller --n is asked for (a quick check)
    kind, parts = _reference_parts(n)
    order = [BLOCK_PARTS[i % len(BLOCK_PARTS)] for i in range(args.warmup + args.steps)]
    warm = _time_parts(parts, order[:args.warmup])
    t0 = time.perf_counter()
    timed = _time_parts(parts, order[args.warmup:])
    wall = time.perf_counter() - t0
    per = {}
    for name in BLOCK_PARTS:
        src = timed.get(name) or warm.get(name)
        per[name] = sum(src) / len(src) if src else None
    if any(v is None for v in per.values()):  # K + W < 7: time the rest once
        rest = [k for k, v in per.items() if v is None]
        for k, v in _time_parts(parts, rest).items():
            per[k] = v[0]
    value = sum(per.values()) * 1e3
    who = ("the reference's own torch modules (xfold.nn.pairformer from baseline/_ref)"
           if kind == "reference" else "the CPU oracle (restated reference torch path)")
    sample = (f"one step = one of the block's 7 sub-modules at N={n} in rotation under CPU "
              f"bf16 autocast, {who}; value = sum of the sub-modules' mean times")
    line = {"impl": "reference", "metric": METRIC, "value": round(value, 1), "unit": UNIT,
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(wall / max(args.steps, 1) * 1e3, 1),
            "higher_is_better": False, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded N(0,1) pair/single, random-init N(0,0.02) weights)",
            "config": {"workload": f"48-block Pairformer trunk, N_token={n}"
                                   + (" (BASELINE config C4)" if n == N_TOKEN else ""),
                       "n_token": n, "blocks": N_BLOCKS, "c_pair": C_PAIR,
                       "c_single": C_SINGLE, "heads_pair": 4, "heads_single": 16, "seed": SEED,
                       "mask": "64-token padded tail", "parallelism": "host CPU"},
            "per_part_ms": {k: round(v * 1e3, 1) for k, v in per.items()},
            "cpu_baseline": {"value": round(value, 1), "unit": UNIT, "cores": threads,
                             "kind": kind, "sample": sample},
            "e2e": {"value": round(value, 1), "unit": UNIT, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------- GPU arm

# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) per launch, from one
# ncu capture of the block's own launches of the same kernels on the same shapes
# (N = 1024: the outgoing contraction and the starting-node triangle attention).
# flash_tri_kernel: 1.0838e9 read + 0.2540e9 written (q, k, v, gate and bias in,
# the gated output out); outgoing contraction gemm_bf16_kernel<256, 4, 0, 0,
# EpiDirect<256>>: 0.5370e9 read + 0.2337e9 written (a and b in, z out): both at
# their algorithmic bytes, no re-reads.
TRAFFIC_BYTES = {"flash_attn": 1.3378e9, "triangle_contraction": 0.7708e9}


def _kernel_roofline(dev, steps: int, peaks: dict) -> dict:
    """Times the triangle-attention flash kernel and the triangle contraction
    GEMM on the block's shapes with CUDA events on the launching stream."""
    import torch

    import oracle
    from xfold_cpu_b200 import native

    n, c, heads, d = N_TOKEN, C_PAIR, 4, 32
    log2e = 1.4426950408889634
    g = torch.Generator(device=dev).manual_seed(11)
    # the operands of the block's triangle attention: q carries log2(e)/sqrt(d),
    # the bias log2(e) (scores in base-2 units), the gate is already squashed
    q = (torch.randn(n, heads, n, d, device=dev, generator=g) * (log2e / d ** 0.5)).bfloat16()
    k = torch.randn(n, heads, n, d, device=dev, generator=g).bfloat16()
    v = torch.randn(n, heads, n, d, device=dev, generator=g).bfloat16()
    bias = (torch.randn(heads, n, n, device=dev, generator=g) * log2e).bfloat16()
    gate = torch.rand(n, n, c, device=dev, generator=g).bfloat16()
    att_out = torch.empty(n, n, c, device=dev, dtype=torch.bfloat16)
    seq = torch.ones(n, device=dev)
    seq[-64:] = 0
    mask = seq[:, None] * seq[None, :]
    a = torch.randn(c, n, n, device=dev, generator=g).bfloat16()
    b = torch.randn(c, n, n, device=dev, generator=g).bfloat16()
    stream = torch.cuda.current_stream(dev)
    results = {}
    for name, fn, flops in (
        ("flash_attn", lambda: native.grid_attention_core(q, k, v, mask, bias, gate, att_out),
         4.0 * heads * n ** 3 * d),
        ("triangle_contraction", lambda: native.gemm(a, b, out_dtype=torch.bfloat16),
         2.0 * c * n ** 3),
    ):
        for _ in range(3):
            fn()
        torch.cuda.synchronize(dev)
        times = []
        for _ in range(max(steps, 5)):
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            fn()
            e1.record(stream)
            e1.synchronize()
            times.append(e0.elapsed_time(e1) * 1e-3)
        t = sum(times) / len(times)
        achieved = flops / t / 1e12
        results[name] = {"bound": "tensor", "achieved": round(achieved, 1),
                         "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                         "frac": round(achieved / peaks["bf16_tflops"], 4),
                         "traffic": TRAFFIC_BYTES[name],
                         "ms_per_launch": round(t * 1e3, 4),
                         "flops_per_launch": flops}
    del q, k, v, bias, gate, att_out, a, b
    return results


def _diffusion_c5(dev, steps: int) -> dict:
    """BASELINE config C5's token transformer: 24 blocks (6 super-blocks of 4),
    N = 768 tokens, c = 768, 16 heads of 48, single cond 384, pair cond 128,
    random init N(0, 0.02), seed 4.  The pair logits are computed once, as the
    reference caches them across denoising steps; one call = the 24 blocks of
    one denoising step, timed eager and as a replayed CUDA graph."""
    import torch

    from xfold_cpu_b200 import _capi
    from xfold_cpu_b200.nn import DiffusionTransformer, init_params_

    n, c = 768, 768
    with torch.inference_mode(False):  # parameters with version counters: weight caches hit
        mod = DiffusionTransformer(c_act=c).eval()
        init_params_(mod, seed=4)
        mod = mod.to(dev)
    g = torch.Generator(device=dev).manual_seed(4)
    act = torch.randn(n, c, device=dev, generator=g)
    cond = torch.randn(n, 384, device=dev, generator=g)
    pair_cond = torch.randn(n, n, 128, device=dev, generator=g)
    mask = torch.ones(n, device=dev)
    stream = torch.cuda.current_stream(dev)
    out = {"n_token": n, "c_act": c, "blocks": 24, "heads": 16, "head_dim": 48,
           "data": "synthetic, random init"}
    with torch.inference_mode():
        logits = mod.pair_logits(pair_cond)
        work = act.clone()

        def eager():
            work.copy_(act)
            mod.run_blocks(work, mask, cond, logits)

        step = mod.capture(act, mask, cond, pair_cond)
        for name, fn in (("eager_ms", eager), ("graph_ms", lambda: step(act, cond))):
            for _ in range(3):
                fn()
            torch.cuda.synchronize(dev)
            l0 = _capi.launch_count()
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            reps = max(steps, 10)
            e0.record(stream)
            for _ in range(reps):
                fn()
            e1.record(stream)
            e1.synchronize()
            out[name] = round(e0.elapsed_time(e1) / reps, 4)
            if name == "eager_ms":
                out["kernel_launches_per_step"] = int((_capi.launch_count() - l0) // reps)
        del step
    return out


ATOM_SUBSETS = 192  # C5: N_atom = 6144 in windows of 32 queries


def _atom_windows(subsets: int, masked_tail: int):
    """Synthetic atom layout of C5: the keys of subset s are the 128 atoms
    centred on its 32 queries (atoms outside [0, N_atom) invalid), the last
    `masked_tail` atoms are padding (queries_mask False), keys_mask is the
    queries mask gathered as the reference's encoder derives it."""
    import torch

    from xfold_cpu_b200.nn import GatherInfo

    rows = subsets * 32
    idx = (torch.arange(subsets)[:, None] * 32 - 48) + torch.arange(128)[None, :]
    valid = (idx >= 0) & (idx < rows)
    idx = torch.where(valid, idx, torch.zeros_like(idx))
    qmask = torch.ones(rows, dtype=torch.bool)
    qmask[rows - masked_tail:] = False
    info = GatherInfo(gather_idxs=idx, gather_mask=valid, input_shape=torch.tensor((subsets, 32)))
    return info, qmask.reshape(subsets, 32), qmask[idx] & valid


def _atom_inputs(subsets: int, seed: int):
    import torch

    g = torch.Generator().manual_seed(seed)
    act = torch.randn(subsets, 32, 128, generator=g)
    qsc = torch.randn(subsets, 32, 128, generator=g)
    pair_cond = torch.randn(subsets, 32, 128, 16, generator=g)
    return act, qsc, pair_cond


def _atom_c5(dev, steps: int) -> dict:
    """BASELINE config C5's atom transformer: N_atom = 6144 (192 windows of 32
    queries x 128 keys), c = 128, 4 heads, 3 blocks, 5 % padded atoms, random
    init N(0, 0.02), seed 4.  One call = DiffusionCrossAttTransformer.forward
    with its pair logits cached (the reference caches them across denoising
    steps): the conditioning of the three blocks and the blocks, timed eager
    and as a replayed CUDA graph.  The encoder and the decoder each make one
    such call per denoising step."""
    import torch

    from xfold_cpu_b200 import _capi
    from xfold_cpu_b200.nn import DiffusionCrossAttTransformer, atom_layout, init_params_

    s = ATOM_SUBSETS
    with torch.inference_mode(False):  # parameters with version counters: weight caches hit
        mod = DiffusionCrossAttTransformer().eval()
        init_params_(mod, seed=4)
        mod = mod.to(dev)
    info, qmask, kmask = _atom_windows(s, (s * 32) // 20)
    act, qsc, pair_cond = (t.to(dev) for t in _atom_inputs(s, 4))
    qmask, kmask = qmask.to(dev), kmask.to(dev)
    stream = torch.cuda.current_stream(dev)
    out = {"n_atom": s * 32, "subsets": s, "queries": 32, "keys": 128, "c_atom": 128, "heads": 4,
           "blocks": 3, "data": "synthetic centred windows, random init"}
    with torch.inference_mode():
        ksc = atom_layout.convert(info, qsc, layout_axes=(-3, -2))
        keys = mod.key_gather(info, s * 32, dev)
        logits = mod.pair_logits(pair_cond)
        work = act.clone()

        def eager():
            work.copy_(act)
            mod.run_blocks(work, qmask, keys, kmask, qsc, ksc, logits)

        step = mod.capture(act, qmask, info, kmask, qsc, ksc, pair_cond)
        for name, fn in (("eager_ms", eager), ("graph_ms", lambda: step(act, qsc, ksc))):
            for _ in range(3):
                fn()
            torch.cuda.synchronize(dev)
            l0 = _capi.launch_count()
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            reps = max(steps, 20)
            e0.record(stream)
            for _ in range(reps):
                fn()
            e1.record(stream)
            e1.synchronize()
            out[name] = round(e0.elapsed_time(e1) / reps, 4)
            if name == "eager_ms":
                out["kernel_launches_per_call"] = int((_capi.launch_count() - l0) // reps)
        del step
    return out


C5_SAMPLES, C5_STEPS = 5, 200


def _c5_sampling(dev, world: int, rank: int) -> dict:
    """BASELINE config C5 end to end on the in-scope modules: 5 samples x 200
    denoising steps, each step = the atom encoder's transformer, the 24-block
    token transformer and the atom decoder's transformer, every one a replayed
    CUDA graph (sizes and init of _diffusion_c5 / _atom_c5; the two atom
    transformers have their own weights).  Samples are spread over the ranks
    by the reference's cyclic schedule (xfold/distributed.py:14-37, samples.py
    work_indices); each step feeds its outputs to the next.  The time is this
    rank's wall on the device; the caller takes the max over ranks."""
    import torch

    from xfold_cpu_b200 import samples
    from xfold_cpu_b200.nn import DiffusionCrossAttTransformer, DiffusionTransformer, init_params_

    n, c, s = 768, 768, ATOM_SUBSETS
    with torch.inference_mode(False):
        tok = DiffusionTransformer(c_act=c).eval()
        init_params_(tok, seed=4)
        enc = DiffusionCrossAttTransformer().eval()
        init_params_(enc, seed=5)
        dec = DiffusionCrossAttTransformer().eval()
        init_params_(dec, seed=6)
        tok, enc, dec = tok.to(dev), enc.to(dev), dec.to(dev)
    g = torch.Generator(device=dev).manual_seed(4)
    act = torch.randn(n, c, device=dev, generator=g)
    cond = torch.randn(n, 384, device=dev, generator=g)
    pair_cond = torch.randn(n, n, 128, device=dev, generator=g)
    mask = torch.ones(n, device=dev)
    info, qmask, kmask = _atom_windows(s, (s * 32) // 20)
    atom_act, qsc, atom_pair = (t.to(dev) for t in _atom_inputs(s, 4))
    qmask, kmask = qmask.to(dev), kmask.to(dev)
    mine = list(samples.work_indices(C5_SAMPLES, rank, world))
    stream = torch.cuda.current_stream(dev)
    with torch.inference_mode():
        from xfold_cpu_b200.nn import atom_layout

        ksc = atom_layout.convert(info, qsc, layout_axes=(-3, -2))
        enc_step = enc.capture(atom_act, qmask, info, kmask, qsc, ksc, atom_pair)
        dec_step = dec.capture(atom_act, qmask, info, kmask, qsc, ksc, atom_pair)
        tok_step = tok.capture(act, mask, cond, pair_cond)

        def one_step(a_atom, a_tok):
            a_atom = enc_step(a_atom, qsc, ksc)
            a_tok = tok_step(a_tok, cond)
            a_atom = dec_step(a_atom, qsc, ksc)
            return a_atom, a_tok

        for _ in range(3):  # warm-up
            one_step(atom_act, act)
        torch.cuda.synchronize(dev)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in mine:
            a_atom, a_tok = atom_act, act
            for _ in range(C5_STEPS):
                a_atom, a_tok = one_step(a_atom, a_tok)
        e1.record(stream)
        e1.synchronize()
        ms = e0.elapsed_time(e1)
        finite = bool(torch.isfinite(a_tok).all()) if mine else True
        del enc_step, dec_step, tok_step
    return {"samples": C5_SAMPLES, "steps_per_sample": C5_STEPS, "samples_this_rank": len(mine),
            "ms": ms, "finite": finite,
            "step": "atom encoder transformer + 24-block token transformer + atom decoder "
                    "transformer, each a replayed CUDA graph",
            "scope": "the in-scope modules of a denoising step (the diffusion head's "
                     "featurisation, atom layout conversions and EDM update are out of scope)"}


EVO_N, EVO_S = 1024, 1024  # the reference's MSA stack: num_msa = 1024 at N_token = 1024


def _evo_inputs(n: int, s: int, seed: int):
    """Synthetic MSA-stack inputs: msa ~ N(0,1) [s, n, 64], pair ~ N(0,1)
    [n, n, 128]; the last 5 % of tokens are padding (masked in every sequence
    and in the pair mask) and 10 % of the other MSA entries are gaps."""
    import torch

    g = torch.Generator().manual_seed(seed)
    msa = torch.randn(s, n, 64, generator=g)
    pair = torch.randn(n, n, 128, generator=g)
    tail = max(1, n // 20)
    msa_mask = (torch.rand(s, n, generator=g) > 0.1).float()
    msa_mask[0] = 1.0
    msa_mask[:, n - tail:] = 0.0
    seq = torch.ones(n)
    seq[n - tail:] = 0.0
    return msa, pair, msa_mask, seq[:, None] * seq[None, :]


def _evoformer(dev, steps: int) -> dict:
    """One Evoformer block of the reference's MSA stack (N_token = 1024,
    num_msa = 1024, c_msa = 64, c_pair = 128, random init N(0, 0.02), seed 5),
    timed eager per block, with a per-operator split from one more pass."""
    import torch

    from xfold_cpu_b200 import _capi
    from xfold_cpu_b200.nn import EvoformerBlock, init_params_

    n, s = EVO_N, EVO_S
    with torch.inference_mode(False):
        blk = EvoformerBlock().eval()
        init_params_(blk, seed=5)
        blk = blk.to(dev)
    msa_h, pair_h, mask_h, pmask_h = _evo_inputs(n, s, 5)
    msa, pair = msa_h.to(dev), pair_h.to(dev)
    mask, pmask = mask_h.to(dev), pmask_h.to(dev)
    stream = torch.cuda.current_stream(dev)
    out = {"n_token": n, "num_msa": s, "c_msa": 64, "c_pair": 128,
           "data": "synthetic, random init, 5 % padded tokens, 10 % MSA gaps"}
    with torch.inference_mode():
        for _ in range(2):
            blk(msa, pair, mask, pmask)
        torch.cuda.synchronize(dev)
        l0 = _capi.launch_count()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        reps = max(steps, 3)
        e0.record(stream)
        for _ in range(reps):
            blk(msa, pair, mask, pmask)
        e1.record(stream)
        e1.synchronize()
        out["ms_per_block"] = round(e0.elapsed_time(e1) / reps, 3)
        out["kernel_launches_per_block"] = int((_capi.launch_count() - l0) // reps)
        parts = [("outer_product_mean", lambda: blk.outer_product_mean.accumulate_(pair, msa, mask)),
                 ("msa_attention", lambda: blk.msa_attention1.accumulate_(msa, mask, pair)),
                 ("msa_transition", lambda: blk.msa_transition.accumulate_(msa))]
        for name, fn in parts:
            fn()
            torch.cuda.synchronize(dev)
            a0 = torch.cuda.Event(enable_timing=True)
            a1 = torch.cuda.Event(enable_timing=True)
            a0.record(stream)
            for _ in range(reps):
                fn()
            a1.record(stream)
            a1.synchronize()
            out[f"{name}_ms"] = round(a0.elapsed_time(a1) / reps, 3)
        if _capi.device_error(clear=True):
            raise RuntimeError("a device wait expired in the Evoformer timing")
    opm_flops = 2 * s * (32 * n) ** 2 + 2 * n * n * 1024 * 128
    out["outer_product_mean_tflops"] = round(opm_flops / (out["outer_product_mean_ms"] * 1e-3) / 1e12, 1)
    return out


def cpu_baseline_evoformer(sample: int = 128, threads: int | None = None) -> dict:
    """The CPU oracle of one Evoformer block at N = num_msa = `sample`,
    float32, scaled to N = num_msa = 1024 by the FLOP ratio."""
    import torch

    import oracle
    from xfold_cpu_b200.nn import EvoformerBlock, init_params_

    if threads:
        torch.set_num_threads(threads)
    blk = EvoformerBlock()
    init_params_(blk, seed=5)
    params = {k: v.detach().clone() for k, v in blk.state_dict().items()}
    msa, pair, mask, pmask = _evo_inputs(sample, sample, 5)
    with torch.inference_mode():
        oracle.evoformer_block(msa, pair, mask, pmask, params)  # warm-up
        t0 = time.perf_counter()
        oracle.evoformer_block(msa, pair, mask, pmask, params)
        dt = time.perf_counter() - t0
    scale = (oracle.evoformer_block_flops(EVO_S, EVO_N)["total"]
             / oracle.evoformer_block_flops(sample, sample)["total"])
    return {"value": round(dt * scale * 1e3, 1), "unit": "ms/block", "cores": torch.get_num_threads(),
            "kind": "port", "sample": (f"1 Evoformer block at N = num_msa = {sample} fp32 (torch CPU "
                                       f"oracle of the reference torch path), {dt:.2f} s, scaled "
                                       f"x{scale:.1f} by FLOPs to {EVO_N}")}


def cpu_baseline_atom(threads: int | None = None) -> dict:
    """The CPU oracle (the reference's torch path restated, float32) of one
    C5 atom-transformer call at full size, on the host's cores."""
    import torch

    import oracle
    from xfold_cpu_b200.nn import DiffusionCrossAttTransformer, init_params_

    if threads:
        torch.set_num_threads(threads)
    s = ATOM_SUBSETS
    mod = DiffusionCrossAttTransformer()
    init_params_(mod, seed=4)
    params = {k: v.detach().clone() for k, v in mod.state_dict().items()}
    info, qmask, kmask = _atom_windows(s, (s * 32) // 20)
    act, qsc, pair_cond = _atom_inputs(s, 4)
    ksc = oracle.atom_layout_convert(info.gather_idxs, info.gather_mask, qsc)
    args = (act, qmask, info.gather_idxs, info.gather_mask, kmask, qsc, ksc, pair_cond, params)
    with torch.inference_mode():
        logits = oracle.cross_pair_logits(pair_cond, params)  # cached, as on the GPU
        oracle.diffusion_cross_att_transformer(*args, logits=logits)  # warm-up
        t0 = time.perf_counter()
        reps = 3
        for _ in range(reps):
            oracle.diffusion_cross_att_transformer(*args, logits=logits)
        dt = (time.perf_counter() - t0) / reps
    return {"value": round(dt * 1e3, 2), "unit": "ms/call", "cores": torch.get_num_threads(),
            "kind": "port", "sample": f"{reps} full C5 atom-transformer calls (pair logits cached), "
                                      "fp32 torch CPU oracle of the reference torch path"}


def run_only(args) -> None:
    """Eager calls of one C5 transformer, for launch lists and captures: the
    same modules and inputs as the extras of the default run."""
    import torch

    from xfold_cpu_b200 import _capi, native
    from xfold_cpu_b200.nn import (DiffusionCrossAttTransformer, DiffusionTransformer,
                                   atom_layout, init_params_)

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    native.check_device(dev)
    if args.only == "evoformer":
        from xfold_cpu_b200.nn import EvoformerBlock

        blk = EvoformerBlock().eval()
        init_params_(blk, seed=5)
        blk = blk.to(dev)
        msa, pair, mask, pmask = (t.to(dev) for t in _evo_inputs(EVO_N, EVO_S, 5))
        with torch.inference_mode():
            for _ in range(args.warmup + args.steps):
                blk(msa, pair, mask, pmask)
            torch.cuda.synchronize(dev)
        print(json.dumps({"only": args.only, "calls": args.warmup + args.steps,
                          "device_error": _capi.device_error(clear=True),
                          "finite": bool(torch.isfinite(pair).all() and torch.isfinite(msa).all())}))
        return
    if args.only == "atom":
        s = ATOM_SUBSETS
        mod = DiffusionCrossAttTransformer().eval()
        init_params_(mod, seed=4)
        mod = mod.to(dev)
        info, qmask, kmask = _atom_windows(s, (s * 32) // 20)
        act, qsc, pair_cond = (t.to(dev) for t in _atom_inputs(s, 4))
        qmask, kmask = qmask.to(dev), kmask.to(dev)
    else:
        n = 768
        mod = DiffusionTransformer(c_act=n).eval()
        init_params_(mod, seed=4)
        mod = mod.to(dev)
        g = torch.Generator(device=dev).manual_seed(4)
        act = torch.randn(n, n, device=dev, generator=g)
        cond = torch.randn(n, 384, device=dev, generator=g)
        pair_cond = torch.randn(n, n, 128, device=dev, generator=g)
        mask = torch.ones(n, device=dev)
    with torch.inference_mode():
        if args.only == "atom":
            ksc = atom_layout.convert(info, qsc, layout_axes=(-3, -2))
            keys = mod.key_gather(info, s * 32, dev)
            logits = mod.pair_logits(pair_cond)
            call = lambda w: mod.run_blocks(w, qmask, keys, kmask, qsc, ksc, logits)
        else:
            logits = mod.pair_logits(pair_cond)
            call = lambda w: mod.run_blocks(w, mask, cond, logits)
        work = act.clone()
        for _ in range(args.warmup + args.steps):
            work.copy_(act)
            call(work)
        torch.cuda.synchronize(dev)
    print(json.dumps({"only": args.only, "calls": args.warmup + args.steps,
                      "device_error": _capi.device_error(clear=True),
                      "finite": bool(torch.isfinite(work).all())}))


def _sharded_parity(dev, blk, pair_h, pair_mask_h, single_h, seq_mask_h, rows, world,
                    exchange) -> dict:
    """Block 0 of the trunk run twice on this rank before the timing: row-sharded
    over the N GPUs (this rank's rows, the exchanges of the timed run) and whole
    on this GPU alone; max |sharded - whole| / max |whole| of the pair update on
    this rank's rows and of the single update, maximum over ranks.  Both
    computations are the CUDA path (no oracle): the check is that sharding
    changes nothing beyond bf16 rounding."""
    import torch
    import torch.distributed as dist

    from xfold_cpu_b200 import sharded

    with torch.inference_mode():
        pm, sm = pair_mask_h.to(dev), seq_mask_h.to(dev)
        whole = pair_h.to(dev)
        s_whole = single_h.to(dev)
        blk(whole, pm, s_whole, sm)
        part0 = pair_h[rows].to(dev)
        part = part0.clone()
        s_part = single_h.to(dev)
        sharded.pairformer_block(blk, [part], pm, s_part, sm, exchange)
        want = whole[rows] - part0
        single0 = single_h.to(dev)
        stats = torch.tensor([(part - part0 - want).abs().max().item(), want.abs().max().item(),
                              (s_part - s_whole).abs().max().item(),
                              (s_whole - single0).abs().max().item()],
                             dtype=torch.float64, device=dev)
        del whole, part, part0, want
    dist.all_reduce(stats, op=dist.ReduceOp.MAX)
    pair_err = stats[0].item() / max(stats[1].item(), 1e-30)
    single_err = stats[2].item() / max(stats[3].item(), 1e-30)
    return {"pair_update_rel_err": round(pair_err, 6), "single_update_rel_err": round(single_err, 6),
            "pair_update_max_abs": round(stats[1].item(), 6),
            "single_update_max_abs": round(stats[3].item(), 6),
            "tolerance": PARITY_TOL, "ok": max(pair_err, single_err) <= PARITY_TOL,
            "what": f"block 0 row-sharded over {world} GPUs vs the same block on one GPU, "
                    "all rows, max over ranks"}


def run_cuda(args) -> None:
    import torch

    world, rank, local = _dist()
    dev = torch.device("cuda", local if torch.cuda.device_count() > local else 0)
    torch.cuda.set_device(dev)
    from xfold_cpu_b200 import _capi, native
    from xfold_cpu_b200.nn import PairformerBlock, init_params_

    native.check_device(dev)
    peaks = _peaks()
    n_tok, n_blocks = args.n, args.blocks
    blocks = []
    for i in range(n_blocks):
        blk = PairformerBlock(c_pair=C_PAIR, c_single=C_SINGLE).eval()
        init_params_(blk, seed=SEED * 1000 + i)
        blocks.append(blk.to(dev))
    pair_h, pair_mask_h, single_h, seq_mask_h = _inputs(n_tok, SEED)
    sharded_parity = None
    single_stream = single_exchange = None
    if world > 1:
        # row-sharded pair: this rank holds rows R_rank of the one N x N trunk
        from xfold_cpu_b200 import sharded

        sharded.check_sharding(n_tok, C_PAIR, world)
        rows = sharded.shard_rows(n_tok, world, rank)
        # peer stores over NVLink by default; XFB_EXCHANGE=collective uses NCCL all-to-all
        exchange = (sharded.ProcessGroupExchange()
                    if os.environ.get("XFB_EXCHANGE", "peer") == "collective"
                    else sharded.PeerExchange())
        sharded_parity = _sharded_parity(dev, blocks[0], pair_h, pair_mask_h, single_h,
                                          seq_mask_h, rows, world, exchange)
        # the single track overlaps the next block's pair operators on its own
        # stream with its own exchange (XFB_SINGLE_OVERLAP=0: in line)
        if (isinstance(exchange, sharded.PeerExchange)
                and os.environ.get("XFB_SINGLE_OVERLAP", "1") == "1"):
            single_stream = torch.cuda.Stream(dev)
            single_exchange = sharded.PeerExchange()
        pair_h = pair_h[rows].contiguous()
    pair_h, pair_mask_h = pair_h.pin_memory(), pair_mask_h.pin_memory()
    single_h, seq_mask_h = single_h.pin_memory(), seq_mask_h.pin_memory()
    pair = pair_h.to(dev)
    single = single_h.to(dev)
    pair_mask = pair_mask_h.to(dev)
    seq_mask = seq_mask_h.to(dev)
    stream = torch.cuda.current_stream(dev)

    def trunk(p, s, pm, sm):
        for blk in blocks:
            if world > 1:
                sharded.pairformer_block(blk, [p], pm, s, sm, exchange,
                                         single_stream=single_stream,
                                         single_exchange=single_exchange)
            else:
                blk(p, pm, s, sm)
        if world > 1 and single_stream is not None:
            torch.cuda.current_stream(dev).wait_stream(single_stream)
        return p, s

    with torch.inference_mode():
        for _ in range(args.warmup):
            trunk(pair, single, pair_mask, seq_mask)
        torch.cuda.synchronize(dev)
        if _capi.device_error(clear=True):
            raise RuntimeError("a device wait expired during warm-up")
        # Row-sharded over N GPUs a block is ~1/N of the GPU work but the same
        # host work (some 25 stage calls, 50 launches), so the trunk is captured
        # into one CUDA graph and replayed: the exchanges' barriers keep their
        # epochs on the device, every rank replays the same graph.
        use_graph = (os.environ.get("XFB_TRUNK_GRAPH", "1" if world > 1 else "0") == "1"
                     and args.warmup > 0)  # the exchanges set up their buffers eagerly
        graph = None
        graph_launches = 0
        if use_graph:
            graph = torch.cuda.CUDAGraph()
            c0 = _capi.launch_count()
            with torch.cuda.graph(graph):
                trunk(pair, single, pair_mask, seq_mask)
            graph_launches = _capi.launch_count() - c0  # kernels in one replay
            torch.cuda.synchronize(dev)
            _barrier(world)

        def step():
            if graph is not None:
                graph.replay()
            else:
                trunk(pair, single, pair_mask, seq_mask)

        # ---- device-resident timing
        sampler = ClockSampler(dev.index if dev.index is not None else 0)
        launches0 = _capi.launch_count()
        _barrier(world)
        torch.cuda.synchronize(dev)
        sampler.start()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            step()
        e1.record(stream)
        torch.cuda.synchronize(dev)
        clocks = sampler.stop()
        _barrier(world)
        launches = (_capi.launch_count() - launches0) // args.steps + graph_launches
        step_ms = _max_over_ranks(e0.elapsed_time(e1) / args.steps, world)

        if args.skip_extras:
            if rank == 0:
                print(json.dumps({"profile_run": True, "n_token": n_tok, "blocks": n_blocks,
                                  "ms_per_block": step_ms / n_blocks, "gpu_launches": int(launches),
                                  "graph": graph is not None}))
            return
        # ---- end-to-end through the module API with host buffers
        out_pair = torch.empty_like(pair_h).pin_memory()
        out_single = torch.empty_like(single_h).pin_memory()
        h2d = sum(t.numel() * t.element_size() for t in (pair_h, single_h, pair_mask_h, seq_mask_h))
        d2h = out_pair.numel() * 4 + out_single.numel() * 4
        _barrier(world)
        torch.cuda.synchronize(dev)
        f0 = torch.cuda.Event(enable_timing=True)
        f1 = torch.cuda.Event(enable_timing=True)
        f0.record(stream)
        for _ in range(args.steps):
            if graph is not None:  # the graph's own input buffers
                pair.copy_(pair_h, non_blocking=True)
                single.copy_(single_h, non_blocking=True)
                pair_mask.copy_(pair_mask_h, non_blocking=True)
                seq_mask.copy_(seq_mask_h, non_blocking=True)
                graph.replay()
                p, s = pair, single
            else:
                p = pair_h.to(dev, non_blocking=True)
                s = single_h.to(dev, non_blocking=True)
                pm = pair_mask_h.to(dev, non_blocking=True)
                sm = seq_mask_h.to(dev, non_blocking=True)
                p, s = trunk(p, s, pm, sm)
            out_pair.copy_(p, non_blocking=True)
            out_single.copy_(s, non_blocking=True)
        f1.record(stream)
        torch.cuda.synchronize(dev)
        e2e_ms = _max_over_ranks(f0.elapsed_time(f1) / args.steps, world)
        if _capi.device_error(clear=True):
            raise RuntimeError("a device wait expired during the timed region")
        finite = bool(torch.isfinite(out_pair).all() and torch.isfinite(out_single).all())

        roof = _kernel_roofline(dev, args.steps, peaks) if rank == 0 else {}
        c5_run = _c5_sampling(dev, world, rank)
        c5_ms = _max_over_ranks(c5_run["ms"], world)
        c5 = _diffusion_c5(dev, args.steps) if rank == 0 and world == 1 else None
        atom = _atom_c5(dev, args.steps) if rank == 0 and world == 1 else None
        evo = _evoformer(dev, args.steps) if rank == 0 and world == 1 else None

    if rank != 0:
        return
    base = cpu_baseline() if world == 1 else None
    parity = block_parity(dev, blocks[0]) if world == 1 and n_tok == N_TOKEN else None
    parity_fp32 = fp32_parity(dev) if world == 1 and n_tok == N_TOKEN else None
    if atom is not None:
        atom["cpu_port"] = cpu_baseline_atom()
    if evo is not None:
        evo["cpu_port"] = cpu_baseline_evoformer()
    dominant = max(roof.values(), key=lambda r: r["ms_per_launch"]) if roof else None
    line = {
        "metric": METRIC, "value": round(step_ms / n_blocks, 4), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(step_ms, 3),
        "higher_is_better": False, "scaling": "strong" if world > 1 else "weak",
        "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) pair/single, random-init N(0,0.02) weights)",
        "config": {"workload": "48-block Pairformer trunk, N_token=1024 (BASELINE config C4)",
                   "trunk_cuda_graph": graph is not None,
                   "n_token": N_TOKEN, "blocks": N_BLOCKS, "c_pair": C_PAIR, "c_single": C_SINGLE,
                   "heads_pair": 4, "heads_single": 16, "seed": SEED, "mask": "64-token padded tail",
                   "l2": "inputs larger than L2 (pair f32 = 512 MiB)",
                   "parallelism": (f"row-sharded pair over {world} GPUs ("
                                   + ("NCCL all-to-all / all-gather"
                                      if os.environ.get("XFB_EXCHANGE", "peer") == "collective"
                                      else ("routed stages (producers store into the peers' "
                                            "receive buffers over NVLink)"
                                            if getattr(exchange, "routes", False)
                                            else "peer-store exchange kernel over NVLink")
                                      + " + " + ("NCCL barrier"
                                                 if os.environ.get("XFB_EXCHANGE_BARRIER") == "nccl"
                                                 else "flag barrier")
                                      + ("; single track on its own stream"
                                         if single_stream is not None else ""))
                                   + ")") if world > 1 else "single GPU"},
        "e2e": {"value": round(e2e_ms / n_blocks, 4), "unit": UNIT, "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h,
                "note": "step = one 48-block trunk pass; host pinned in/out"
                        + ("; bytes per rank (its pair rows, the masks, the single copy)"
                           if world > 1 else "")},
        "gpu_launches": int(launches),
        "roofline": ({**{k: v for k, v in dominant.items()},
                      "kernel": [k for k, v in roof.items() if v is dominant][0],
                      "peak_source": peaks["source"]} if dominant else None),
        "kernels": roof,
        "clocks": clocks,
        "cpu_baseline": base,
        "finite": finite,
        "parity": parity,
        "parity_fp32": parity_fp32,
        "sharded_parity": sharded_parity,
        "extras": {"diffusion_c5_5x200": {**c5_run, "ms": round(c5_ms, 1), "gpus": world,
                                          "ms_note": "max over ranks of each rank's samples"},
                   **({"diffusion_transformer_c5": c5, "atom_transformer_c5": atom,
                       "evoformer_block": evo} if c5 else {})},
    }
    print(json.dumps(line), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("cuda", "reference"), default="cuda")
    ap.add_argument("--blocks", type=int, default=N_BLOCKS,
                    help="trunk depth (48 for the metric; fewer only for profiling)")
    ap.add_argument("--n", type=int, default=N_TOKEN,
                    help="N_token (1024 for the metric; smaller only for profiling)")
    ap.add_argument("--skip-extras", action="store_true",
                    help="profiling mode: no e2e pass, kernel roofline or CPU baseline")
    ap.add_argument("--only", choices=("atom", "diffusion", "evoformer"), default=None,
                    help="run only the C5 atom or token transformer: --warmup + --steps eager "
                         "calls, one JSON line (a profiling target)")
    args = ap.parse_args()
    if args.only:
        run_only(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_cuda(args)
    try:
        import torch.distributed as dist

        if dist.is_initialized():
            dist.destroy_process_group()
    except Exception:
        pass


if __name__ == "__main__":
    main()
