"""The INT8 overlay loader (QuantizedWeights::{load,get}, src/cpu/quantized.rs:
239-370) and the safetensors checks it stands on (src/checkpoint.rs:101-166).

CPU tests drive the library's host-only validation (uocr_overlay_check): the
reference writer's golden overlay (tests/golden/overlay, made by
tests/golden/make_overlay_golden.py with tools/quantize.py), the fixtures and
rejections of tests/quantized_loader.rs and tests/checkpoint.rs, manifest and
metadata rules, and SHA-256 against hashlib.  GPU tests load overlays into
device memory and compute through them, and check the package's writer
(GPU quantization) byte for byte against the reference writer's output.
"""
import hashlib
import json
import os
import shutil
import struct

import numpy as np
import pytest

import oracle
from conftest import ROOT
from helpers import bits_equal

GOLDEN = os.path.join(ROOT, "tests", "golden", "overlay")
G_SRC = os.path.join(GOLDEN, "source.safetensors")
G_OV = os.path.join(GOLDEN, "overlay.safetensors")


def write_st(path, header, data=b""):
    """safetensors bytes: u64 LE header length, JSON header, payload
    (tests/quantized_loader.rs:8-14)."""
    raw = header if isinstance(header, bytes) else json.dumps(header, separators=(",", ":")).encode()
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(raw)) + raw + data)


def sha(path):
    return hashlib.sha256(open(path, "rb").read()).hexdigest()


def reference_fixture(d):
    """tests/quantized_loader.rs:15-35: W = [1, -2] (F32 source), overlay
    bytes [1, 254] with scale 1.0; returns (source, overlay) paths."""
    src = os.path.join(d, "source.safetensors")
    write_st(src, {"lm_head.weight": {"dtype": "F32", "shape": [1, 2], "data_offsets": [0, 8]}},
             struct.pack("<2f", 1.0, -2.0))
    h = sha(src)
    ov = os.path.join(d, "q.safetensors")
    write_st(ov, {"__metadata__": {"format": "uocr-q8-block32-v1", "block_size": "32",
                                   "source_sha256": h},
                  "lm_head.weight": {"dtype": "I8", "shape": [1, 2], "data_offsets": [0, 2]},
                  "lm_head.weight.q8_scales": {"dtype": "F32", "shape": [1, 1],
                                               "data_offsets": [2, 6]}},
             bytes([1, 254]) + struct.pack("<f", 1.0))
    write_manifest(ov, h)
    return src, ov


def write_manifest(ov, source_hash, **override):
    m = {"schema_version": 1, "format": "uocr-q8-block32-v1", "block_size": 32,
         "source_sha256": source_hash, "output_sha256": sha(ov), "matrix_count": 1,
         "bytes": os.path.getsize(ov)}
    m.update(override)
    with open(os.path.splitext(ov)[0] + ".json", "w") as f:
        json.dump(m, f)


def split(path):
    b = open(path, "rb").read()
    n = struct.unpack("<Q", b[:8])[0]
    return json.loads(b[8:8 + n]), b[8 + n:]


def read_tensors(path):
    """name -> float32/int8 array of a safetensors file (test reader)."""
    header, data = split(path)
    header.pop("__metadata__", None)
    out = {}
    for name, d in header.items():
        raw = np.frombuffer(data[d["data_offsets"][0]:d["data_offsets"][1]], np.uint8)
        if d["dtype"] == "F32":
            v = raw.view("<f4")
        elif d["dtype"] == "F16":
            v = raw.view("<f2").astype(np.float32)
        elif d["dtype"] == "BF16":
            v = (raw.view("<u2").astype(np.uint32) << 16).view(np.float32)
        elif d["dtype"] == "I8":
            v = raw.view(np.int8)
        else:
            continue
        out[name] = v.reshape(d["shape"])
    return out


def kind_of(fn):
    import uocr_q8
    with pytest.raises(uocr_q8.OcrError) as e:
        fn()
    return e.value.kind


# ---- CPU: host validation through the library ------------------------------

@pytest.mark.parametrize("n", [0, 1, 55, 56, 63, 64, 65, 119, 120, 1000, 3 * 1024 * 1024 + 19])
def test_sha256_matches_hashlib(tmp_path, n):
    from uocr_q8.overlay import sha256_file
    # tests/checkpoint.rs:58-60 pattern (i * 113) as u8
    data = (np.arange(n, dtype=np.int64) * 113 % 256).astype(np.uint8).tobytes()
    p = tmp_path / "f.bin"
    p.write_bytes(data)
    assert sha256_file(p) == hashlib.sha256(data).hexdigest()


def test_sha256_portable_rounds_match_hashlib(tmp_path):
    """The portable rounds (the form used where the CPU lacks the SHA
    extensions), forced in a child process."""
    import subprocess
    import sys
    code = (
        "import hashlib, sys, numpy as np\n"
        "from uocr_q8.overlay import sha256_file\n"
        "for n in (0, 55, 56, 64, 119, 1 << 20):\n"
        "    d = (np.arange(n) * 113 % 256).astype(np.uint8).tobytes()\n"
        f"    p = {str(tmp_path / 'x')!r}\n"
        "    open(p, 'wb').write(d)\n"
        "    assert sha256_file(p) == hashlib.sha256(d).hexdigest(), n\n")
    env = dict(os.environ, UOCR_SHA_PORTABLE="1",
               PYTHONPATH=os.pathsep.join([os.path.join(ROOT, "unlimited-ocr-kernel_b200"), ROOT]))
    subprocess.run([sys.executable, "-c", code], check=True, env=env)


def test_golden_overlay_accepted():
    from uocr_q8.overlay import check
    man = json.load(open(os.path.join(GOLDEN, "overlay.json")))
    n, dev_bytes = check(G_OV, G_SRC)
    assert n == man["matrix_count"] == 7
    ov = read_tensors(G_OV)
    expect = 0
    for name in sorted(k for k in ov if not k.endswith(".q8_scales")):
        for arr in (ov[name], ov[name + ".q8_scales"]):
            expect = (expect + arr.nbytes + 255) // 256 * 256
    assert dev_bytes == expect


def test_golden_overlay_is_the_oracle_quantization():
    """The reference writer's bytes equal the oracle's Int8Matrix::quantize
    of the source matrices (F32, F16 and BF16 sources, short tails, a zero
    row): pins the oracle to the reference's writer."""
    src, ov = read_tensors(G_SRC), read_tensors(G_OV)
    names = [k for k in ov if not k.endswith(".q8_scales")]
    assert len(names) == 7
    for name in names:
        m = oracle.quantize(src[name].astype(np.float32))
        assert np.array_equal(m.w, ov[name]), name
        assert bits_equal(m.s, ov[name + ".q8_scales"]), name


def test_reference_fixture_accepted(tmp_path):
    from uocr_q8.overlay import check
    src, ov = reference_fixture(str(tmp_path))
    assert check(ov, src)[0] == 1


def test_corruption_and_wrong_source_rejected(tmp_path):
    """tests/quantized_loader.rs:51-63."""
    from uocr_q8.overlay import check
    src, ov = reference_fixture(str(tmp_path))
    original = open(ov, "rb").read()
    flipped = bytearray(original)
    flipped[-1] ^= 1
    open(ov, "wb").write(bytes(flipped))
    assert kind_of(lambda: check(ov, src)) == "Format"
    open(ov, "wb").write(original)
    wrong = str(tmp_path / "other.safetensors")
    write_st(wrong, {"lm_head.weight": {"dtype": "F32", "shape": [1, 2], "data_offsets": [0, 8]}},
             bytes(8))
    assert kind_of(lambda: check(ov, wrong)) == "Format"
    assert check(ov, src)[0] == 1


@pytest.mark.parametrize("invalid,kind", [
    ("version", "Format"), ("scale", "Numerical"), ("shape", "Format"),
    ("dtype", "Format"), ("range", "Format"), ("missing", "Format"),
    ("negative_scale", "Numerical"), ("scales_shape", "Format"), ("scales_dtype", "Format"),
])
def test_authenticated_but_invalid_overlay_rejected(tmp_path, invalid, kind):
    """tests/quantized_loader.rs:66-107 (the manifest re-signed after each
    change), plus negative scales and wrong scale shape/dtype."""
    from uocr_q8.overlay import check
    src, ov = reference_fixture(str(tmp_path))
    header, data = split(ov)
    data = bytearray(data)
    if invalid == "version":
        header["__metadata__"]["format"] = "future"
    elif invalid == "scale":
        data[2:6] = struct.pack("<f", float("nan"))
    elif invalid == "negative_scale":
        data[2:6] = struct.pack("<f", -1.0)
    elif invalid == "shape":
        header["lm_head.weight"]["shape"] = [2, 1]
    elif invalid == "dtype":
        header["lm_head.weight"]["dtype"] = "F16"
    elif invalid == "range":
        data[0] = 128
    elif invalid == "missing":
        del header["lm_head.weight.q8_scales"]
    elif invalid == "scales_shape":
        header["lm_head.weight.q8_scales"]["shape"] = [1, 1, 1]
    elif invalid == "scales_dtype":
        header["lm_head.weight.q8_scales"]["dtype"] = "I8"
        header["lm_head.weight.q8_scales"]["shape"] = [4]
    write_st(ov, header, bytes(data))
    write_manifest(ov, sha(src))
    assert kind_of(lambda: check(ov, src)) == kind


def test_negative_zero_scale_accepted(tmp_path):
    """from_parts accepts -0.0 scales (src/cpu/quantized.rs:31-35)."""
    from uocr_q8.overlay import check
    src, ov = reference_fixture(str(tmp_path))
    header, data = split(ov)
    write_st(ov, header, data[:2] + struct.pack("<f", -0.0))
    write_manifest(ov, sha(src))
    assert check(ov, src)[0] == 1


@pytest.mark.parametrize("case,kind", [
    ("missing_manifest", "Io"), ("bad_json", "Json"), ("missing_field", "Json"),
    ("string_count", "Json"), ("float_count", "Json"), ("schema_2", "Format"),
    ("block_16", "Format"), ("bytes", "Format"), ("upper_hash", "Format"),
    ("count_2", "Format"), ("meta_block_size", "Format"), ("meta_source", "Format"),
    ("no_metadata", "Format"), ("duplicate_field", "Json"),
])
def test_manifest_and_metadata_rules(tmp_path, case, kind):
    """Manifest decoding and the version/metadata check
    (src/cpu/quantized.rs:306-322)."""
    from uocr_q8.overlay import check
    src, ov = reference_fixture(str(tmp_path))
    h = sha(src)
    mpath = os.path.splitext(ov)[0] + ".json"
    if case == "missing_manifest":
        os.remove(mpath)
    elif case == "bad_json":
        open(mpath, "w").write("{\"schema_version\": 1,")
    elif case == "missing_field":
        m = json.load(open(mpath))
        del m["output_sha256"]
        json.dump(m, open(mpath, "w"))
    elif case == "string_count":
        write_manifest(ov, h, matrix_count="1")
    elif case == "float_count":
        write_manifest(ov, h, matrix_count=1.0)
    elif case == "schema_2":
        write_manifest(ov, h, schema_version=2)
    elif case == "block_16":
        write_manifest(ov, h, block_size=16)
    elif case == "bytes":
        write_manifest(ov, h, bytes=os.path.getsize(ov) + 1)
    elif case == "upper_hash":
        write_manifest(ov, h.upper())
    elif case == "count_2":
        write_manifest(ov, h, matrix_count=2)
    elif case in ("meta_block_size", "meta_source", "no_metadata"):
        header, data = split(ov)
        if case == "meta_block_size":
            header["__metadata__"]["block_size"] = "32.0"
        elif case == "meta_source":
            header["__metadata__"]["source_sha256"] = "0" * 64
        else:
            del header["__metadata__"]
        write_st(ov, header, data)
        write_manifest(ov, h)
    elif case == "duplicate_field":
        m = json.dumps({"schema_version": 1, "format": "uocr-q8-block32-v1", "block_size": 32,
                        "source_sha256": h, "output_sha256": sha(ov), "matrix_count": 1,
                        "bytes": os.path.getsize(ov)})
        open(mpath, "w").write(m[:-1] + ",\"matrix_count\":1}")
    assert kind_of(lambda: check(ov, src)) == kind


def test_unknown_manifest_fields_ignored(tmp_path):
    from uocr_q8.overlay import check
    src, ov = reference_fixture(str(tmp_path))
    write_manifest(ov, sha(src), producer="anything", extra=[1, 2, {"a": None}])
    assert check(ov, src)[0] == 1


def test_matrix_set_rules(tmp_path):
    """Eligible names (src/cpu/quantized.rs:262-301) and the matrix set check
    (:330-336): every eligible source matrix must be in the overlay and the
    overlay must hold nothing else."""
    from uocr_q8.overlay import check
    src, ov = reference_fixture(str(tmp_path))
    header = {"lm_head.weight": {"dtype": "F32", "shape": [1, 2], "data_offsets": [0, 8]},
              "model.norm.weight": {"dtype": "F32", "shape": [2], "data_offsets": [8, 16]},
              "model.layers.x.mlp.gate_proj.weight": {"dtype": "F32", "shape": [1, 2],
                                                      "data_offsets": [16, 24]},
              "model.layers.1.mlp.gate.weight": {"dtype": "F32", "shape": [1, 2],
                                                 "data_offsets": [24, 32]},
              "model.layers.1.self_attn.q_norm.weight": {"dtype": "F32", "shape": [1, 2],
                                                         "data_offsets": [32, 40]}}
    write_st(src, header, struct.pack("<2f", 1.0, -2.0) + bytes(32))
    header2, data2 = split(ov)
    header2["__metadata__"]["source_sha256"] = sha(src)
    write_st(ov, header2, data2)
    write_manifest(ov, sha(src))
    assert check(ov, src)[0] == 1  # none of the extra names is eligible
    header["model.layers.7.mlp.experts.0.up_proj.weight"] = {
        "dtype": "F32", "shape": [1, 2], "data_offsets": [40, 48]}
    write_st(src, header, struct.pack("<2f", 1.0, -2.0) + bytes(40))
    header2["__metadata__"]["source_sha256"] = sha(src)
    write_st(ov, header2, data2)
    write_manifest(ov, sha(src))
    assert kind_of(lambda: check(ov, src)) == "Format"


def test_ineligible_source_dtype_rejected(tmp_path):
    """The source matrix must be BF16, F16 or F32 (src/cpu/quantized.rs:346)."""
    from uocr_q8.overlay import check
    src, ov = reference_fixture(str(tmp_path))
    write_st(src, {"lm_head.weight": {"dtype": "I64", "shape": [1, 2], "data_offsets": [0, 16]}},
             bytes(16))
    header, data = split(ov)
    header["__metadata__"]["source_sha256"] = sha(src)
    write_st(ov, header, data)
    write_manifest(ov, sha(src))
    assert kind_of(lambda: check(ov, src)) == "Format"


@pytest.mark.parametrize("header,kind", [
    # tests/checkpoint.rs:27-33
    (b'{"x":{"dtype":"BF16","shape":[3],"data_offsets":[0,6]}}', "Format"),
    (b'{"x":{"dtype":"F32","shape":[1],"data_offsets":[0,4]},'
     b'"y":{"dtype":"F32","shape":[1],"data_offsets":[0,4]}}', "Format"),
    (b'{"x":{"dtype":"F32","shape":[18446744073709551615,2],"data_offsets":[0,4]}}', "Format"),
    (b'{"x":{"dtype":"F32","shape":[1],"data_offsets":[4,0]}}', "Format"),
    (b'{"x":{"dtype":"UNKNOWN","shape":[1],"data_offsets":[0,4]}}', "Json"),
    # tests/checkpoint.rs:45-50
    (b'{"x":{"dtype":"F32","shape":[2],"data_offsets":[0,4]}}', "Format"),
    (b'{"x":{"dtype":"BF16","shape":[1],"data_offsets":[0,2]}}', "Format"),
    # decoding rules of the header
    (b'{"x":{"dtype":"F32","shape":[1],"data_offsets":[0,4]},"__metadata__":{"a":1}}', "Json"),
    (b'{"x":{"dtype":"F32","shape":[-1],"data_offsets":[0,4]}}', "Json"),
    (b'{"x":{"dtype":"F32","shape":[1],"data_offsets":[0,4,8]}}', "Json"),
    (b'{"x":{"dtype":"F32","shape":[1]}}', "Json"),
    (b'[1,2]', "Json"),
    (b'{"x":{"dtype":"F32","shape":[1],"data_offsets":[0,4]}', "Json"),
    (b'{"x":{"dtype":"F32","shape":[1],"data_offsets":[0,4]}} x', "Json"),
    (b'{"\xff":{"dtype":"F32","shape":[1],"data_offsets":[0,4]}}', "Json"),
])
def test_checkpoint_rejections(tmp_path, header, kind):
    """Checkpoint::open rejections (tests/checkpoint.rs:25-52), seen through
    the loader's source argument."""
    from uocr_q8.overlay import check
    src = str(tmp_path / "bad.safetensors")
    write_st(src, header, bytes(4))
    assert kind_of(lambda: check(G_OV, src)) == kind


def test_checkpoint_header_length_rules(tmp_path):
    from uocr_q8.overlay import check
    p = str(tmp_path / "h.safetensors")
    open(p, "wb").write(struct.pack("<Q", 2 ** 64 - 1))  # tests/checkpoint.rs:35-37
    assert kind_of(lambda: check(G_OV, p)) == "Format"
    open(p, "wb").write(b"\x01\x02")  # shorter than the length field
    assert kind_of(lambda: check(G_OV, p)) == "Format"
    open(p, "wb").write(struct.pack("<Q", 100_000_001) + b"{}")
    assert kind_of(lambda: check(G_OV, p)) == "Format"
    assert kind_of(lambda: check(G_OV, str(tmp_path / "absent"))) == "Io"


def test_checkpoint_accepts_sequence_descriptors_and_escapes(tmp_path):
    """A descriptor given as a sequence, escaped names, unknown descriptor
    keys and white space padding (as the reference's writer pads the header
    to 8 bytes) decode like the reference's typed decoding."""
    from uocr_q8.overlay import check
    src, ov = reference_fixture(str(tmp_path))
    raw = (b'{"lm_head.weight":["F32",[1,2],[0,8]],'
           b'"model.\\u006eorm.weight":{"dtype":"F32","shape":[1],"data_offsets":[8,12],"x":null}}'
           + b" " * 5)
    write_st(src, raw, struct.pack("<3f", 1.0, -2.0, 1.0))
    header, data = split(ov)
    header["__metadata__"]["source_sha256"] = sha(src)
    write_st(ov, header, data)
    write_manifest(ov, sha(src))
    assert check(ov, src)[0] == 1


def test_null_arguments():
    import uocr_q8._lib as L
    lib = L.load()
    assert lib.uocr_overlay_check(None, None, None, None) == 11
    assert lib.uocr_overlay_count(None) == 0
    assert lib.uocr_overlay_name(None, 0) is None
    assert lib.uocr_overlay_free(None) == 0


# ---- GPU: device-resident overlays ----------------------------------------

@pytest.mark.gpu
def test_reference_fixture_computes(ctx, tmp_path):
    """tests/quantized_loader.rs:37-50: linear([3, 4]) = [-5]."""
    from uocr_q8.overlay import QuantizedWeights
    src, ov = reference_fixture(str(tmp_path))
    q = QuantizedWeights.load(ov, src, ctx)
    m = q.get("lm_head.weight")
    assert m is not None and (m.rows, m.cols) == (1, 2)
    y = m.linear(np.array([[3.0, 4.0]], np.float32))
    assert y.tolist() == [[-5.0]]
    assert q.get("model.norm.weight") is None
    assert len(q) == 1 and q.names() == ["lm_head.weight"]
    q.free()


@pytest.mark.gpu
def test_invalid_overlay_allocates_nothing(ctx, tmp_path):
    import torch
    from uocr_q8.overlay import QuantizedWeights
    src, ov = reference_fixture(str(tmp_path))
    header, data = split(ov)
    write_st(ov, header, bytes([128]) + data[1:])
    write_manifest(ov, sha(src))
    torch.cuda.synchronize()
    before = torch.cuda.mem_get_info(ctx.device)[0]
    assert kind_of(lambda: QuantizedWeights.load(ov, src, ctx)) == "Format"
    assert torch.cuda.mem_get_info(ctx.device)[0] >= before - (2 << 20)


@pytest.mark.gpu
def test_golden_overlay_on_device(ctx):
    """The reference writer's overlay, loaded: bytes on the device equal the
    file, and every matrix computes like the oracle (linear: FP32 tolerance;
    linear_dynamic_int8: bit-exact)."""
    from uocr_q8.overlay import QuantizedWeights
    from helpers import rel_err, terms_abs
    q = QuantizedWeights.load(G_OV, G_SRC, ctx)
    ov = read_tensors(G_OV)
    names = sorted(k for k in ov if not k.endswith(".q8_scales"))
    assert q.names() == names
    rng = np.random.default_rng(7)
    for name in names:
        m = q.get(name)
        w, s = m.download()
        assert np.array_equal(w, ov[name]) and bits_equal(s, ov[name + ".q8_scales"]), name
        om = oracle.Matrix(w, s)
        x = rng.standard_normal((3, m.cols)).astype(np.float32)
        y = m.linear(x)
        assert rel_err(y, oracle.linear(om, x), terms_abs(w, s, x)) <= 1e-4, name
        for r in range(3):
            assert bits_equal(m.linear_dynamic_int8(x[r:r + 1]),
                              oracle.linear_dynamic_int8(om, x[r:r + 1])), name
    q.free()


@pytest.mark.gpu
def test_overlay_views_on_tensor_core_paths(ctx, tmp_path):
    """Overlay matrices feed the tensor-core kernels (256-byte aligned views):
    a batch of 64 rows through a 256 x 1280 expert-shaped matrix."""
    import torch
    from uocr_q8.overlay import QuantizedWeights, write_overlay
    from helpers import rel_err, terms_abs
    rng = np.random.default_rng(11)
    src = str(tmp_path / "src.safetensors")
    a = (rng.standard_normal((256, 1280)) * 0.05).astype(np.float32)
    b = (rng.standard_normal((384, 1280)) * 0.05).astype(np.float32)
    write_st(src, {"model.layers.3.mlp.experts.0.up_proj.weight":
                   {"dtype": "F32", "shape": [256, 1280], "data_offsets": [0, a.nbytes]},
                   "model.layers.3.mlp.experts.1.up_proj.weight":
                   {"dtype": "F32", "shape": [384, 1280],
                    "data_offsets": [a.nbytes, a.nbytes + b.nbytes]}},
             a.tobytes() + b.tobytes())
    ov = str(tmp_path / "ov.safetensors")
    write_overlay(src, ov, ctx)
    q = QuantizedWeights.load(ov, src, ctx)
    for name, ref in (("model.layers.3.mlp.experts.0.up_proj.weight", a),
                      ("model.layers.3.mlp.experts.1.up_proj.weight", b)):
        m = q.get(name)
        om = oracle.quantize(ref)
        w, s = m.download()
        assert np.array_equal(w, om.w) and bits_equal(s, om.s)
        x = rng.standard_normal((64, 1280)).astype(np.float32)
        y = m.linear_device(torch.from_numpy(x).cuda(ctx.device)).cpu().numpy()
        assert rel_err(y, oracle.linear(om, x), terms_abs(w, s, x)) <= 1e-4
        yd = m.linear_device(torch.from_numpy(x).cuda(ctx.device), dynamic=True).cpu().numpy()
        assert bits_equal(yd, oracle.linear_dynamic_int8(om, x))
    q.free()


@pytest.mark.gpu
def test_writer_matches_reference_writer(ctx, tmp_path):
    """The package's writer (GPU quantization) reproduces the reference
    writer's overlay and manifest byte for byte, and refuses to overwrite."""
    from uocr_q8.overlay import write_overlay
    src = str(tmp_path / "source.safetensors")
    shutil.copyfile(G_SRC, src)
    out = str(tmp_path / "overlay.safetensors")
    write_overlay(src, out, ctx)
    assert open(out, "rb").read() == open(G_OV, "rb").read()
    assert open(str(tmp_path / "overlay.json")).read() == \
        open(os.path.join(GOLDEN, "overlay.json")).read()
    with pytest.raises(FileExistsError):
        write_overlay(src, out, ctx)


@pytest.mark.gpu
def test_writer_rejects_like_reference_writer(ctx, tmp_path):
    """tests/python/test_quantize.py:30-35 (integer source) and nonfinite
    values: ValueError, nothing published."""
    from uocr_q8.overlay import quantize_file
    src = str(tmp_path / "s.safetensors")
    out = tmp_path / "o.safetensors"
    write_st(src, {"lm_head.weight": {"dtype": "I64", "shape": [2, 3], "data_offsets": [0, 48]}},
             bytes(48))
    with pytest.raises(ValueError):
        quantize_file(src, out, ctx)
    assert not out.exists()
    write_st(src, {"lm_head.weight": {"dtype": "F32", "shape": [1, 2], "data_offsets": [0, 8]}},
             struct.pack("<2f", 1.0, float("inf")))
    with pytest.raises(ValueError):
        quantize_file(src, out, ctx)
    assert not out.exists()
    assert sorted(os.listdir(tmp_path)) == ["s.safetensors"]
