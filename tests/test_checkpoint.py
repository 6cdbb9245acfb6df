"""Checkpoint record stream (xfold/params.py:39-95, 213-256): parsing against a
stream the reference's own encoder wrote (tests/golden/make_checkpoint_golden.py)
and what its read_records returned; file selection; errors; and, on the GPU,
the upload through xfb_gather_bytes bit for bit."""

import pathlib
import struct

import numpy as np
import pytest
import torch

from xfold_cpu_b200 import checkpoint

GOLDEN = pathlib.Path(__file__).resolve().parent / "golden"


def _encode(scope, name, arr: np.ndarray) -> bytes:
    """The record format of encode_record (xfold/params.py:39-54)."""
    s, n, d = scope.encode(), name.encode(), str(arr.dtype).encode()
    buf = np.ascontiguousarray(arr).tobytes("C")
    return (struct.pack("<5i", len(s), len(n), len(d), arr.ndim, len(buf)) + s + n + d
            + struct.pack(f"<{arr.ndim}i", *arr.shape) + buf)


def _host_values(blob: bytes, rec: checkpoint.Record) -> np.ndarray:
    if rec.nbytes == 0:
        return np.zeros(rec.shape, dtype=np.float32)
    t = torch.frombuffer(bytearray(blob[rec.offset:rec.offset + rec.nbytes]),
                         dtype=checkpoint.DTYPES[rec.dtype])
    return t.reshape(rec.shape).float().numpy()


def test_parse_matches_reference_reader():
    blob = (GOLDEN / "checkpoint_records.bin").read_bytes()
    want = np.load(GOLDEN / "checkpoint_records.npz")
    recs = checkpoint.parse_records(blob)
    assert [f"{r.scope}/{r.name}" for r in recs] == list(want.keys())
    for r in recs:
        ref = want[f"{r.scope}/{r.name}"]
        assert r.shape == ref.shape and r.dtype == str(ref.dtype)
        np.testing.assert_array_equal(_host_values(blob, r), ref.astype(np.float32))


def test_parse_errors():
    good = _encode("a", "b", np.arange(6, dtype=np.float32).reshape(2, 3))
    with pytest.raises(checkpoint.RecordError):
        checkpoint.parse_records(good + b"\x01\x02")  # incomplete header
    with pytest.raises(checkpoint.RecordError):
        checkpoint.parse_records(good[:-1])  # incomplete payload
    bad = bytearray(good)
    struct.pack_into("<i", bad, 12, 3)  # shape rank 3 for a 2-d record: sizes disagree
    with pytest.raises((checkpoint.RecordError, RuntimeError)):
        checkpoint.parse_records(bytes(bad))
    odd = _encode("a", "b", np.zeros(3, dtype=np.int64))
    with pytest.raises(KeyError):  # the reference's dtype map has no int64
        checkpoint.parse_records(odd)
    assert checkpoint.parse_records(b"") == []
    empty = checkpoint.parse_records(_encode("e", "rows", np.zeros((0, 4), np.float32)))
    assert empty[0].shape == (0, 4) and empty[0].nbytes == 0


def test_select_model_files(tmp_path):
    for name in ("af3.bin.2", "af3.bin.10", "af3.bin.1", "notes.txt"):
        (tmp_path / name).write_bytes(b"")
    files, compressed = checkpoint.select_model_files(tmp_path)
    assert [f.name for f in files] == ["af3.bin.1", "af3.bin.2", "af3.bin.10"] and not compressed
    (tmp_path / "other.bin.zst").write_bytes(b"")
    files, compressed = checkpoint.select_model_files(tmp_path, "other")
    assert [f.name for f in files] == ["other.bin.zst"] and compressed
    with pytest.raises(FileNotFoundError):
        checkpoint.select_model_files(tmp_path, "missing")


def test_compressed_needs_zstandard(tmp_path):
    try:
        import zstandard  # noqa: F401
        pytest.skip("zstandard is installed")
    except ImportError:
        pass
    (tmp_path / "m.bin.zst").write_bytes(b"\x28\xb5\x2f\xfd")
    with pytest.raises(RuntimeError, match="zstandard"):
        checkpoint._read_stream([tmp_path / "m.bin.zst"], True)


@pytest.mark.gpu
def test_upload_matches_host_records(tmp_path):
    """Golden stream split over two files plus larger arrays at odd offsets:
    every device view equals the host decode, and starts 256-byte aligned."""
    rng = np.random.default_rng(3)
    extra = b"".join(_encode(f"s{i}", "w", rng.standard_normal(shape).astype(dt))
                     for i, (shape, dt) in enumerate([((513, 129), np.float32), ((7,), np.uint8),
                                                      ((33, 65), np.float16), ((0, 8), np.float32),
                                                      ((1000,), np.float32)]))
    blob = (GOLDEN / "checkpoint_records.bin").read_bytes() + extra
    cut = len(blob) // 3
    (tmp_path / "m.bin.1").write_bytes(blob[:cut])
    (tmp_path / "m.bin.2").write_bytes(blob[cut:])
    files, compressed = checkpoint.select_model_files(tmp_path)
    got = checkpoint.load_to_device(files, compressed, "cuda")
    recs = checkpoint.parse_records(blob)
    assert list(got) == [f"{r.scope}/{r.name}" for r in recs]
    for r in recs:
        t = got[f"{r.scope}/{r.name}"]
        assert t.is_cuda and t.dtype == checkpoint.DTYPES[r.dtype] and tuple(t.shape) == r.shape
        if r.nbytes:
            assert t.data_ptr() % 256 == 0
        np.testing.assert_array_equal(t.float().cpu().numpy(), _host_values(blob, r))
