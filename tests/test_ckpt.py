"""Merged-INT8 checkpoint reader (csrc/ckpt.cu), on the CPU.

* Round trips through shards written here in the safetensors layout: every
  dtype the reference reads (src/safetensors.rs:22-38), metadata, several
  shards.
* The header checks of the reference's TensorIndex::add_shard
  (src/safetensors.rs:112-181), one malformed shard per check.
* Where the reference's own fixture checkpoints are mounted (this build
  container), the reader's view of them equals the golden vectors that
  tests/golden/make_golden.py extracted with the Python safetensors reader.
"""
import json
import os
import struct

import numpy as np
import pytest

from doantotnghiepmoe_b200 import Checkpoint, MoeError
from doantotnghiepmoe_b200 import _lib
from tests.helpers import write_safetensors

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
# the reference checkout: MOE_REFERENCE_ROOT, or a `reference` directory
# beside this repository (present only where the reference is mounted)
_REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
FIXTURES = os.path.join(os.environ.get("MOE_REFERENCE_ROOT",
                                       os.path.join(os.path.dirname(_REPO), "reference")),
                        "tests", "fixtures")


def test_round_trip_all_dtypes_two_shards(tmp_path):
    rng = np.random.default_rng(3)
    a = rng.integers(-128, 128, size=(3, 5), dtype=np.int8)
    b = rng.integers(0, 256, size=(7,), dtype=np.uint8)
    c = rng.standard_normal((2, 3, 4)).astype(np.float32)
    d = rng.standard_normal((6,)).astype(np.float16)
    e = (rng.standard_normal((4, 4)).astype(np.float32).view(np.uint32) >> 16).astype(np.uint16)
    write_safetensors(tmp_path / "model-00000.safetensors",
                      [("x.i8", "I8", a), ("x.u8", "U8", b), ("x.f32", "F32", c)],
                      metadata={"format": "pt", "note": "é\\\"q\""})
    write_safetensors(tmp_path / "model-00001.safetensors",
                      [("y.f16", "F16", d), ("y.bf16", "BF16", e), ("y.scalar", "F32",
                                                                   np.float32(2.5).reshape(()))])
    ck = Checkpoint(str(tmp_path))
    assert len(ck) == 6
    assert ck.info("x.i8") == ("I8", (3, 5), 15)
    assert ck.info("y.bf16") == ("BF16", (4, 4), 32)
    assert ck.info("y.scalar") == ("F32", (), 4)
    assert np.array_equal(ck.read("x.i8"), a)
    assert np.array_equal(ck.read("x.u8"), b)
    assert np.array_equal(ck.read("x.f32").view(np.uint32), c.view(np.uint32))
    assert np.array_equal(ck.read("y.f16").view(np.uint16), d.view(np.uint16))
    assert np.array_equal(ck.read("y.bf16"), e)
    with pytest.raises(MoeError):
        ck.info("missing")
    ck.close()


def _raw_shard(path, header: bytes, payload: bytes):
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(header)))
        f.write(header)
        f.write(payload)


def _desc(dtype, shape, b, e):
    return {"dtype": dtype, "shape": shape, "data_offsets": [b, e]}


BAD = {
    "zero_header_length": (b"", b""),
    "not_an_object": (b'["x"]', b""),
    "unknown_dtype": (json.dumps({"t": _desc("F64", [1], 0, 8)}).encode(), bytes(8)),
    "unknown_field": (json.dumps({"t": {**_desc("U8", [1], 0, 1), "x": 1}}).encode(), bytes(1)),
    "missing_field": (json.dumps({"t": {"dtype": "U8", "shape": [1]}}).encode(), bytes(1)),
    "offsets_disagree_with_shape": (json.dumps({"t": _desc("F32", [2], 0, 4)}).encode(), bytes(4)),
    "past_end_of_file": (json.dumps({"t": _desc("U8", [8], 0, 8)}).encode(), bytes(4)),
    "gap": (json.dumps({"a": _desc("U8", [2], 0, 2), "b": _desc("U8", [2], 3, 5)}).encode(),
            bytes(5)),
    "overlap": (json.dumps({"a": _desc("U8", [2], 0, 2), "b": _desc("U8", [2], 1, 3)}).encode(),
                bytes(3)),
    "unindexed_tail": (json.dumps({"a": _desc("U8", [2], 0, 2)}).encode(), bytes(3)),
    "duplicate_name": (b'{"a": {"dtype": "U8", "shape": [1], "data_offsets": [0, 1]}, '
                       b'"a": {"dtype": "U8", "shape": [1], "data_offsets": [1, 2]}}', bytes(2)),
    "metadata_not_strings": (json.dumps({"__metadata__": {"k": 1}}).encode(), b""),
    "negative_number": (b'{"a": {"dtype": "U8", "shape": [-1], "data_offsets": [0, 0]}}', b""),
    "trailing_garbage": (json.dumps({"a": _desc("U8", [1], 0, 1)}).encode() + b" x", bytes(1)),
}


@pytest.mark.parametrize("case", sorted(BAD))
def test_malformed_shard_rejected(tmp_path, case):
    header, payload = BAD[case]
    _raw_shard(tmp_path / "m.safetensors", header, payload)
    with pytest.raises(MoeError) as ei:
        Checkpoint(str(tmp_path))
    assert ei.value.status == _lib.MOE_ERR_INVALID
    assert ei.value.message  # the reason is reported


def test_header_length_past_file_and_no_shards(tmp_path):
    with open(tmp_path / "m.safetensors", "wb") as f:
        f.write(struct.pack("<Q", 1 << 20))
        f.write(b"{}")
    with pytest.raises(MoeError):
        Checkpoint(str(tmp_path))
    empty = tmp_path / "empty"
    empty.mkdir()
    with pytest.raises(MoeError) as ei:
        Checkpoint(str(empty))
    assert "no .safetensors" in ei.value.message


def test_duplicate_across_shards(tmp_path):
    x = np.zeros(4, np.uint8)
    write_safetensors(tmp_path / "a.safetensors", [("t", "U8", x)])
    write_safetensors(tmp_path / "b.safetensors", [("t", "U8", x)])
    with pytest.raises(MoeError) as ei:
        Checkpoint(str(tmp_path))
    assert "duplicate" in ei.value.message


FIXTURE_NAMES = [("olmoe", "unnormalized-mha"), ("olmoe", "normalized-gqa"),
                 ("qwen3moe", "gqa-headdim"), ("qwen3moe", "many-experts"),
                 ("qwen3moe", "bf16-dense")]


@pytest.mark.parametrize("family,name", FIXTURE_NAMES)
def test_reference_fixture_checkpoints(family, name):
    """The reference's fixture models, read by this reader, give the layers
    the golden vectors hold (experts, scales, router bits)."""
    d = os.path.join(FIXTURES, family, name)
    if not os.path.isdir(d):
        pytest.skip("reference fixtures are not mounted here")
    z = np.load(os.path.join(GOLDEN, f"fixture_{family}_{name}.npz"))
    ck = Checkpoint(d)
    E = int(z["E"])
    for l in range(int(z["n_layers"])):
        r = ck.read(f"model.layers.{l}.mlp.gate.weight")
        want = z[f"l{l}_router"]
        if int(z["router_bf16"]):
            assert ck.info(f"model.layers.{l}.mlp.gate.weight")[0] == "BF16"
            assert np.array_equal(r, want.view(np.uint16))
        else:
            assert np.array_equal(r.view(np.uint32), want.view(np.uint32))
        for e in range(E):
            w = ck.read(f"model.layers.{l}.mlp.experts.{e}.merged_weight")
            s = ck.read(f"model.layers.{l}.mlp.experts.{e}.qs")
            assert np.array_equal(w, z[f"l{l}_experts"][e])
            assert np.array_equal(s.view(np.uint32), z[f"l{l}_scales"][e].view(np.uint32))
