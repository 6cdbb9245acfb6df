"""Writes tests/golden/checkpoint_records.{bin,npz}: a small parameter record
stream encoded by the reference's own `encode_record` (xfold/params.py:39-54)
and what its `read_records` (:66-95) returns for it.

Run from the repository root with the reference checkout importable:
    PYTHONPATH=<reference checkout> python tests/golden/make_checkpoint_golden.py
The reference module imports `zstandard` at the top (only its compressed
reader uses it); when the module is absent a placeholder module stands in, and
the uncompressed path is what this script exercises.  No zero-size array is
included: the reference's reader takes `payload[-0:]` (the whole payload) for
one and fails.
"""

import io
import pathlib
import sys
import types

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent


def main() -> None:
    try:
        import zstandard  # noqa: F401
    except ImportError:
        sys.modules["zstandard"] = types.ModuleType("zstandard")
    from xfold import params

    rng = np.random.default_rng(7)
    arrays = [
        ("diffuser/evoformer/pair_norm", "scale", rng.standard_normal((128,)).astype(np.float32)),
        ("diffuser/evoformer/trimul", "weights", rng.standard_normal((3, 5, 7)).astype(np.float32)),
        ("diffuser/head", "half", rng.standard_normal((4, 6)).astype(np.float16)),
        ("diffuser/odd", "bytes", rng.integers(0, 255, (7,), dtype=np.uint8)),
        ("diffuser/scalar", "value", np.array(2.5, dtype=np.float32)),
        ("__meta__", "__identifier__", np.frombuffer(b"synthetic-v1", dtype=np.uint8).copy()),
    ]
    blob = b"".join(params.encode_record(s, n, a) for s, n, a in arrays)
    (HERE / "checkpoint_records.bin").write_bytes(blob)
    expected = {}
    for scope, name, arr in params.read_records(io.BytesIO(blob)):
        expected[f"{scope}/{name}"] = arr.numpy()
    np.savez(HERE / "checkpoint_records.npz", **expected)
    print(f"{len(blob)} bytes, {len(expected)} records")


if __name__ == "__main__":
    main()
