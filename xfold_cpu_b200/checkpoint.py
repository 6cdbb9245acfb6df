"""Parameter checkpoint upload to the GPU.

The reference reads its AF3 parameter file record by record on the host
(xfold/params.py:66-95 `_read_record` / `read_records`, over the concatenated
files of `_MultiFileIO` :98-185, optionally through a zstd stream reader
:188-197) and builds one CPU tensor per record, which the model then copies to
the device tensor by tensor.  Here the whole (decompressed) stream is read
into one pinned host buffer, copied to the device with a single transfer, and
the library's `xfb_gather_bytes` kernel scatters the record payloads into a
device arena where each array starts on a 256-byte boundary; every parameter
is a typed view of that arena.  Record parsing follows `_read_record`: a
'<5i' header (scope, name, dtype and shape lengths and the payload size),
the three strings, the int32 shape and the little-endian payload; a short
header or payload raises RecordError.  File selection follows
`select_model_files` (:213-240).
"""

from __future__ import annotations

import ctypes
import pathlib
import re
import struct
from dataclasses import dataclass

import torch

from . import _capi

DTYPES = {"float32": torch.float32, "bfloat16": torch.bfloat16, "float16": torch.float16,
          "uint8": torch.uint8}
ALIGN = 256
_HEADER = struct.Struct("<5i")


class RecordError(Exception):
    """Error reading a record (xfold/params.py:35-36)."""


@dataclass(frozen=True)
class Record:
    scope: str
    name: str
    dtype: str
    shape: tuple[int, ...]
    offset: int   # payload byte offset in the stream
    nbytes: int


def parse_records(buf) -> list[Record]:
    """Index of every record in a byte buffer (bytes / memoryview / numpy)."""
    mv = memoryview(buf).cast("B")
    out, pos, end = [], 0, len(mv)
    while pos < end:
        if end - pos < _HEADER.size:
            raise RecordError(f"Incomplete header: {end - pos} < {_HEADER.size}")
        sl, nl, dl, rank, nb = _HEADER.unpack_from(mv, pos)
        pos += _HEADER.size
        need = sl + nl + dl + 4 * rank + nb
        if min(sl, nl, dl, rank, nb) < 0 or end - pos < need:
            raise RecordError(f"Incomplete payload: {end - pos} < {need}")
        scope = bytes(mv[pos:pos + sl]).decode("utf-8")
        name = bytes(mv[pos + sl:pos + sl + nl]).decode("utf-8")
        dtype = bytes(mv[pos + sl + nl:pos + sl + nl + dl]).decode("utf-8")
        shape = struct.unpack_from(f"<{rank}i", mv, pos + sl + nl + dl)
        off = pos + sl + nl + dl + 4 * rank
        if dtype not in DTYPES:
            raise KeyError(dtype)
        item = torch.empty((), dtype=DTYPES[dtype]).element_size()
        count = 1
        for d in shape:
            count *= d
        if count * item != nb:  # the reference's reshape fails the same way
            raise RuntimeError(f"shape '{list(shape)}' is invalid for input of size "
                               f"{nb // item} ({scope}/{name})")
        out.append(Record(scope, name, dtype, tuple(shape), off, nb))
        pos = off + nb
    return out


def _read_stream(files: list[pathlib.Path], is_compressed: bool) -> torch.Tensor:
    """The concatenated (decompressed) contents of `files` in pinned host memory."""
    if not files:
        raise ValueError("At least one checkpoint file is required.")
    if is_compressed:
        try:
            import zstandard
        except ImportError as error:
            raise RuntimeError("compressed (.zst) checkpoints need the zstandard module") from error
        raw = b"".join(pathlib.Path(f).read_bytes() for f in files)
        data = zstandard.ZstdDecompressor().stream_reader(raw).read()
        blob = torch.empty(len(data), dtype=torch.uint8, pin_memory=True)
        blob.numpy()[:] = memoryview(data)
        return blob
    sizes = [pathlib.Path(f).stat().st_size for f in files]
    blob = torch.empty(sum(sizes), dtype=torch.uint8, pin_memory=True)
    view, pos = blob.numpy(), 0
    for f, size in zip(files, sizes):
        with open(f, "rb") as handle:
            got = handle.readinto(memoryview(view[pos:pos + size]))
        if got != size:
            raise OSError("Checkpoint file changed or ended before its recorded size.")
        pos += size
    return blob


def load_to_device(files, is_compressed: bool = False,
                   device: torch.device | str = "cuda") -> dict[str, torch.Tensor]:
    """{"scope/name": device tensor} of every record, like
    get_alphafold3_params (xfold/params.py:245-256) but on `device`."""
    device = torch.device(device)
    if device.type != "cuda":
        raise ValueError("load_to_device uploads to a CUDA device")
    files = [pathlib.Path(f) for f in (files if isinstance(files, (list, tuple)) else [files])]
    blob = _read_stream(files, is_compressed)
    records = parse_records(blob.numpy())
    spans, pos = [], 0
    for r in records:
        spans.append((r.offset, pos, r.nbytes))
        pos += -(-r.nbytes // ALIGN) * ALIGN
    arena = torch.empty(max(pos, ALIGN), dtype=torch.uint8, device=device)
    if records:
        src = blob.to(device, non_blocking=True)
        host_spans = torch.tensor(spans, dtype=torch.int64)
        dev_spans = host_spans.to(device)
        stream = torch.cuda.current_stream(device).cuda_stream
        _capi.call("xfb_gather_bytes", src.data_ptr(), src.numel(), arena.data_ptr(),
                   arena.numel(), dev_spans.data_ptr(),
                   ctypes.cast(host_spans.data_ptr(), ctypes.c_void_p), len(records), stream)
        torch.cuda.current_stream(device).synchronize()  # src / spans are released on return
    out = {}
    for r, (_, dst, nb) in zip(records, spans):
        out[f"{r.scope}/{r.name}"] = arena[dst:dst + nb].view(DTYPES[r.dtype]).view(r.shape)
    return out


def select_model_files(model_dir: pathlib.Path, model_name: str | None = None
                       ) -> tuple[list[pathlib.Path], bool]:
    """The model files of a directory and whether they are zstd-compressed
    (xfold/params.py:213-240: same patterns, same part ordering)."""
    files = [f for f in pathlib.Path(model_dir).iterdir() if f.is_file()]
    for pattern, compressed in (
        (r"(?P<model_name>.*)\.(?P<part>[0-9]+)\.bin\.zst$", True),
        (r"(?P<model_name>.*)\.bin\.zst\.(?P<part>[0-9]+)$", True),
        (r"(?P<model_name>.*)\.(?P<part>[0-9]+)\.bin$", False),
        (r"(?P<model_name>.*)\.bin\.(?P<part>[0-9]+)$", False),
        (r"(?P<model_name>.*)\.bin\.zst$", True),
        (r"(?P<model_name>.*)\.bin$", False),
    ):
        rx = re.compile(pattern)
        models: dict[str, list[pathlib.Path]] = {}
        for f in files:
            m = rx.fullmatch(f.name)
            if m:
                models.setdefault(m.group("model_name"), []).append(f)
        models = {k: sorted(v, key=lambda p: int(rx.fullmatch(p.name).groupdict().get("part") or 0))
                  for k, v in models.items()}
        if model_name is not None:
            if model_name in models:
                return models[model_name], compressed
        elif models:
            if len(models) > 1:
                raise RuntimeError(f"Multiple models matched in {model_dir}")
            return next(iter(models.values())), compressed
    raise FileNotFoundError(f"No models matched in {model_dir}")
