"""Host-side logic on the CPU: checkpoint layout parity with the reference
modules, the backend switch, weight caches and argument validation."""

from pathlib import Path

import numpy as np
import pytest
import torch

from xfold_cpu_b200 import native
from xfold_cpu_b200.fastnn import WeightCache, config
from xfold_cpu_b200.nn import (DiffusionTransition, GridSelfAttention, PairformerBlock, SelfAttention,
                               Transition, TriangleMultiplication, init_params_)

GOLDEN = Path(__file__).resolve().parent / "golden"


def golden_params(name):
    data = np.load(GOLDEN / f"{name}.npz")
    return {k[6:]: data[k].shape for k in data.files if k.startswith("param:")}


@pytest.mark.parametrize("name,module", [
    ("triangle_outgoing", lambda: TriangleMultiplication(16, _outgoing=True)),
    ("grid_attention_ending", lambda: GridSelfAttention(16, 4, transpose=True)),
    ("transition", lambda: Transition(16, 4)),
    ("self_attention_plain", lambda: SelfAttention(32, 8, 4, use_single_cond=False)),
    ("self_attention_conditioned", lambda: SelfAttention(32, 8, 4, use_single_cond=True)),
    ("diffusion_transition", lambda: DiffusionTransition(16, 8, use_single_cond=True)),
    ("pairformer_block", lambda: PairformerBlock(n_heads=4, c_pair=16, c_single=32, n_heads_pair=4)),
])
def test_state_dict_matches_reference_layout(name, module):
    """Same parameter names and shapes as the reference modules, so reference
    state_dicts / checkpoint imports load unchanged."""
    ref = golden_params(name)
    mine = {k: tuple(v.shape) for k, v in module().state_dict().items()}
    assert mine == {k: tuple(v) for k, v in ref.items()}


def test_reference_state_dict_loads():
    data = np.load(GOLDEN / "pairformer_block.npz")
    sd = {k[6:]: torch.from_numpy(data[k]) for k in data.files if k.startswith("param:")}
    block = PairformerBlock(n_heads=4, c_pair=16, c_single=32, n_heads_pair=4)
    block.load_state_dict(sd, strict=True)


def test_backend_switch_rejects_other_implementations():
    mod = Transition(16)
    old = config.gated_linear_unit_implementation
    config.gated_linear_unit_implementation = "cpp"
    try:
        with pytest.raises(ValueError, match="only the 'cuda' backend"):
            mod(torch.randn(2, 16))
    finally:
        config.gated_linear_unit_implementation = old


def test_cuda_backend_refuses_cpu_tensors():
    mod = TriangleMultiplication(16)
    with pytest.raises(ValueError, match="CUDA tensors"):
        mod(torch.randn(4, 4, 16), torch.ones(4, 4))


def test_inference_only_guard():
    x = torch.randn(4, 8, requires_grad=True)
    with pytest.raises((RuntimeError, ValueError)):
        native.linear(x, torch.randn(8, 8))


def test_weight_cache_reuses_until_the_weight_changes():
    calls = []
    cache = WeightCache()
    w = torch.randn(4, 4)

    def build(t):
        calls.append(1)
        return t * 2

    a = cache.get((w,), build)
    assert cache.get((w,), build) is a and len(calls) == 1
    with torch.no_grad():
        w.add_(1)
    b = cache.get((w,), build)
    assert b is not a and len(calls) == 2
    torch.testing.assert_close(b, w * 2)


def test_init_params_is_deterministic_and_follows_the_recipe():
    a = PairformerBlock(c_pair=16, c_single=32, n_heads=4, n_heads_pair=4)
    b = PairformerBlock(c_pair=16, c_single=32, n_heads=4, n_heads_pair=4)
    init_params_(a, seed=7)
    init_params_(b, seed=7)
    for (ka, va), (kb, vb) in zip(a.state_dict().items(), b.state_dict().items()):
        assert ka == kb and torch.equal(va, vb)
    w = a.triangle_multiplication_outgoing.projection.weight
    assert abs(w.std().item() - 0.02) < 0.003
    assert torch.equal(a.triangle_multiplication_outgoing.left_norm_input.weight, torch.ones(16))


def test_af3_compat_mirrors_the_reference_argument_checks():
    """xfold_cpu_b200.af3_compat (the af3_kernels._C stand-in) refuses what the
    reference's native extension refuses, before any device work: non-device
    tensors, VNNI2-packed weights, non-positive tile sizes."""
    import pytest
    import torch

    from xfold_cpu_b200 import af3_compat

    x = torch.zeros(4, 8)
    with pytest.raises(RuntimeError, match="CUDA"):
        af3_compat.linear(x, torch.zeros(8, 8))
    with pytest.raises(RuntimeError, match="VNNI2"):
        af3_compat.gated_linear_unit(x, torch.zeros(8, 16), weight_packed=True)
    with pytest.raises(RuntimeError, match="VNNI2"):
        af3_compat.triangle_multiplication(*([None] * 11), weights_packed=True)
    assert af3_compat.packed_weight_api == 0
    assert af3_compat.load_extension() is af3_compat


def test_bench_reference_arm_prints_its_line(tmp_path):
    """`bench.py --impl reference` end to end on the CPU at a small N (the
    driver runs it at the default N = 1024): one JSON line with the reference
    arm's keys."""
    import json
    import subprocess
    import sys
    from pathlib import Path

    root = Path(__file__).resolve().parents[1]
    out = subprocess.run([sys.executable, str(root / "bench.py"), "--impl", "reference",
                          "--steps", "7", "--warmup", "1", "--n", "64"],
                         capture_output=True, text=True, timeout=600, cwd=str(tmp_path))
    assert out.returncode == 0, out.stderr[-2000:]
    line = json.loads(out.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["value"] > 0
    assert line["e2e"]["value"] == line["value"] and line["cpu_baseline"]["kind"] in (
        "reference", "port")
    assert set(line["per_part_ms"]) == {"triangle_multiplication_outgoing",
                                        "triangle_multiplication_incoming", "pair_attention1",
                                        "pair_attention2", "pair_transition",
                                        "single_attention", "single_transition"}
