"""The ``uocr-q8-block32-v1`` INT8 overlay: loader and writer.

``QuantizedWeights`` mirrors the reference's loader (src/cpu/quantized.rs:
239-370): ``QuantizedWeights.load(path, source)`` validates the overlay at
``path`` against the source checkpoint and its manifest (``path`` with the
extension ``.json``) and makes every matrix device-resident;
``get(name)`` returns the ``Int8Matrix`` or None.  All validation and the
upload run in the CUDA library (uocr_overlay_load); ``check`` runs the same
validation without a device.

``quantize_file`` mirrors the reference's writer (tools/quantize.py:37-88):
the same eligible names, file layout, header bytes and manifest, with the
quantization itself run on the GPU (uocr_q8_quantize, bit-identical to
``quantize_blocks`` / ``Int8Matrix::quantize``).  ``write_overlay`` also
writes the manifest beside the overlay, as the tool's ``main`` does
(tools/quantize.py:91-98).
"""
from __future__ import annotations

import ctypes
import hashlib
import json
import os
import re
import struct
import tempfile
from pathlib import Path
from typing import Dict, List, Optional, Tuple

import numpy as np

from . import BLOCK, GpuContext, Int8Matrix, _check, default_context, lib

FORMAT = "uocr-q8-block32-v1"
SUFFIX = ".q8_scales"
# tools/quantize.py:16 (ASCII digits, as the Rust loader's usize parse wants)
MATRIX = re.compile(r"^(?:lm_head|model\.layers\.[0-9]+\.(?:self_attn\.[qkvo]_proj|mlp\."
                    r"(?:(?:experts\.[0-9]+|shared_experts)\.)?(?:gate|up|down)_proj))\.weight$")


def _path(p) -> bytes:
    return os.fsencode(os.fspath(p))


class QuantizedWeights:
    """Validated, device-resident overlay matrices (name -> Int8Matrix)."""

    def __init__(self, handle, ctx: GpuContext):
        self._h = handle
        self.ctx = ctx
        self._views: Dict[str, Int8Matrix] = {}

    @classmethod
    def load(cls, path, source, ctx: Optional[GpuContext] = None) -> "QuantizedWeights":
        """QuantizedWeights::load(path, &Checkpoint::open(source))."""
        ctx = ctx or default_context()
        h = ctypes.c_void_p()
        _check(lib().uocr_overlay_load(ctx.handle, _path(path), _path(source), ctypes.byref(h)))
        return cls(h, ctx)

    def get(self, name: str) -> Optional[Int8Matrix]:
        if name in self._views:
            return self._views[name]
        m = ctypes.c_void_p()
        _check(lib().uocr_overlay_get(self._h, name.encode(), ctypes.byref(m)))
        if not m.value:
            return None
        view = Int8Matrix(m, self.ctx, keepalive=self, owned=False)
        self._views[name] = view
        return view

    def names(self) -> List[str]:
        L = lib()
        return [L.uocr_overlay_name(self._h, i).decode() for i in range(len(self))]

    def __len__(self) -> int:
        return int(lib().uocr_overlay_count(self._h))

    def __contains__(self, name: str) -> bool:
        return self.get(name) is not None

    def device_bytes(self) -> int:
        return int(lib().uocr_overlay_device_bytes(self._h))

    def free(self) -> None:
        if getattr(self, "_h", None):
            for v in self._views.values():
                v._h = None
            self._views.clear()
            lib().uocr_overlay_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


def check(path, source) -> Tuple[int, int]:
    """Every check of QuantizedWeights::load, without a device: (matrix count,
    device bytes a load takes).  Raises OcrError like load."""
    n, b = ctypes.c_size_t(), ctypes.c_size_t()
    _check(lib().uocr_overlay_check(_path(path), _path(source), ctypes.byref(n), ctypes.byref(b)))
    return n.value, b.value


def sha256_file(path) -> str:
    """Lowercase hex SHA-256 of a file, computed by the library."""
    out = ctypes.create_string_buffer(65)
    _check(lib().uocr_sha256_file(_path(path), out))
    return out.value.decode()


# ---- writer ---------------------------------------------------------------

_DTYPES = {"F32": 4, "F16": 2, "BF16": 2}


def _read_header(path: Path):
    with open(path, "rb") as f:
        n = struct.unpack("<Q", f.read(8))[0]
        header = json.loads(f.read(n))
    header.pop("__metadata__", None)
    return header, 8 + n


def _matrix_f32(mm: np.memmap, start: int, desc, rows: slice) -> np.ndarray:
    """Rows of a source matrix as float32 (exact for F32, F16 and BF16)."""
    r, c = desc["shape"]
    esz = _DTYPES[desc["dtype"]]
    lo, hi = rows.start, rows.stop
    raw = mm[start + desc["data_offsets"][0] + lo * c * esz:
             start + desc["data_offsets"][0] + hi * c * esz]
    if desc["dtype"] == "F32":
        v = raw.view("<f4")
    elif desc["dtype"] == "F16":
        v = raw.view("<f2").astype(np.float32)
    else:
        v = (raw.view("<u2").astype(np.uint32) << 16).view(np.float32)
    return np.ascontiguousarray(v.reshape(hi - lo, c), dtype=np.float32)


def _sha256(path: Path) -> str:
    digest = hashlib.sha256()
    with open(path, "rb") as stream:
        for block in iter(lambda: stream.read(8 * 1024 * 1024), b""):
            digest.update(block)
    return digest.hexdigest()


def quantize_file(source, output, ctx: Optional[GpuContext] = None,
                  chunk_rows: int = 65536) -> dict:
    """Write the overlay of ``source`` to ``output``; returns the manifest.

    Same contract as tools/quantize.py:37-88: a distinct, not yet existing
    output; the source left intact and checked unchanged; the file published
    by a hard link from a temporary only when complete; ValueError for an
    ineligible source (no matrices, a dtype other than F32/F16/BF16, a
    matrix that is not 2-D and nonempty, nonfinite values, scale underflow).
    """
    from . import OcrError
    ctx = ctx or default_context()
    source, output = Path(source).resolve(), Path(output).resolve()
    if source == output or chunk_rows <= 0:
        raise ValueError("use a distinct output and positive chunk size")
    if output.exists():
        raise FileExistsError(output)
    source_hash = _sha256(source)
    output.parent.mkdir(parents=True, exist_ok=True)
    fd, temporary = tempfile.mkstemp(prefix=output.name + ".", suffix=".tmp", dir=output.parent)
    os.close(fd)
    try:
        tensors, data_start = _read_header(source)
        names = sorted(n for n in tensors if MATRIX.fullmatch(n))
        if not names:
            raise ValueError("no supported decoder matrices")
        header = {"__metadata__": {"format": FORMAT, "block_size": str(BLOCK),
                                   "source_sha256": source_hash}}
        offset = 0
        for name in names:
            d = tensors[name]
            if d["dtype"] not in _DTYPES:
                raise ValueError(f"unsupported source dtype: {name}")
            shape = list(d["shape"])
            if len(shape) != 2 or 0 in shape:
                raise ValueError(f"invalid matrix {name}")
            rows, cols = shape
            blocks = (cols + BLOCK - 1) // BLOCK
            header[name] = {"dtype": "I8", "shape": shape,
                            "data_offsets": [offset, offset + rows * cols]}
            offset += rows * cols
            header[name + SUFFIX] = {"dtype": "F32", "shape": [rows, blocks],
                                     "data_offsets": [offset, offset + rows * blocks * 4]}
            offset += rows * blocks * 4
        raw = json.dumps(header, separators=(",", ":")).encode()
        raw += b" " * ((-len(raw)) % 8)
        start = 8 + len(raw)
        mm = np.memmap(source, dtype=np.uint8, mode="r")
        with open(temporary, "wb") as stream:
            stream.write(struct.pack("<Q", len(raw)))
            stream.write(raw)
            stream.truncate(start + offset)
            for name in names:
                rows, cols = header[name]["shape"]
                blocks = (cols + BLOCK - 1) // BLOCK
                for row in range(0, rows, chunk_rows):
                    hi = min(row + chunk_rows, rows)
                    values = _matrix_f32(mm, data_start, tensors[name], slice(row, hi))
                    try:
                        m = Int8Matrix.quantize(values, ctx)
                    except OcrError as e:
                        raise ValueError(f"{name}: {e.message}") from None
                    q, s = m.download()
                    m.free()
                    stream.seek(start + header[name]["data_offsets"][0] + row * cols)
                    stream.write(q.tobytes())
                    stream.seek(start + header[name + SUFFIX]["data_offsets"][0] + row * blocks * 4)
                    stream.write(s.astype("<f4", copy=False).tobytes())
            stream.flush()
            os.fsync(stream.fileno())
        del mm
        if _sha256(source) != source_hash:
            raise ValueError("source changed during export")
        result = {"schema_version": 1, "format": FORMAT, "block_size": BLOCK,
                  "source_sha256": source_hash, "output_sha256": _sha256(Path(temporary)),
                  "matrix_count": len(names), "bytes": Path(temporary).stat().st_size}
        os.link(temporary, output)
        return result
    finally:
        Path(temporary).unlink(missing_ok=True)


def write_overlay(source, output, ctx: Optional[GpuContext] = None) -> dict:
    """quantize_file plus the manifest at ``output`` with suffix .json."""
    result = quantize_file(source, output, ctx)
    Path(output).with_suffix(".json").write_text(json.dumps(result, indent=2) + "\n")
    return result


__all__ = ["QuantizedWeights", "check", "sha256_file", "quantize_file", "write_overlay",
           "FORMAT", "SUFFIX", "MATRIX"]
