"""Checkpoint parsing on the CPU (kvb_checkpoint_open / _tensor / the argument
checks of _load_rows; reference engine/src/model/weights.rs:112-230): shards
are indexed, later shards replace earlier names, and every malformed input is
an error with a message, never a crash.  Loads that copy run in the GPU tests."""
import ctypes as C
import json
import os
import struct

import numpy as np
import pytest
import torch

import st_util as S
from kvasir_b200.gpu import CheckpointError, CheckpointIoError, ShapeError
from kvasir_b200.weights import Checkpoint


def _shard(tmp_path, name, tensors, metadata=None):
    S.write(os.path.join(tmp_path, name), tensors, metadata)


def test_index_and_shard_order(tmp_path):
    rng = np.random.default_rng(1)
    _shard(tmp_path, "model-00001-of-00002.safetensors",
           {"a": S.f32(rng.normal(size=6), (2, 3)), "shared": S.f16(np.ones(4), (4,)),
            "café.weight": S.bf16(np.arange(5, dtype=np.uint16), (5,))},
           metadata={"format": "pt"})
    _shard(tmp_path, "model-00002-of-00002.safetensors",
           {"b": S.bf16(np.zeros(8, np.uint16), (2, 2, 2)), "shared": S.f32(np.ones(3), (3,)),
            "i": ("I32", (2,), np.array([1, 2], "<i4").tobytes())})
    (tmp_path / "notes.txt").write_text("not a shard")
    with Checkpoint(str(tmp_path)) as ck:
        assert len(ck) == 5
        assert ck.info("a") == ("F32", (2, 3))
        assert ck.info("b") == ("BF16", (2, 2, 2))
        assert ck.info("café.weight") == ("BF16", (5,))
        assert ck.info("shared") == ("F32", (3,))  # the later shard wins
        assert ck.info("i") == ("other", (2,))
        with pytest.raises(CheckpointError, match="missing tensor nope"):
            ck.info("nope")


def test_missing_directory_and_no_shards(tmp_path):
    with pytest.raises(CheckpointIoError):
        Checkpoint(str(tmp_path / "absent"))
    with pytest.raises(CheckpointError, match="no .safetensors files"):
        Checkpoint(str(tmp_path))


@pytest.mark.parametrize("blob,msg", [
    (b"\x01\x02", "shorter than the 8-byte header length"),
    (struct.pack("<Q", 1000) + b"{}", "header length 1000 exceeds the file"),
    (struct.pack("<Q", 6) + b'{"a":}', "malformed header JSON"),
    (struct.pack("<Q", 2) + b"[]", "malformed header JSON"),
])
def test_malformed_headers(tmp_path, blob, msg):
    (tmp_path / "x.safetensors").write_bytes(blob)
    with pytest.raises(CheckpointError, match=msg):
        Checkpoint(str(tmp_path))


def _raw_shard(tmp_path, header: dict, data: bytes):
    text = json.dumps(header).encode()
    (tmp_path / "x.safetensors").write_bytes(struct.pack("<Q", len(text)) + text + data)


@pytest.mark.parametrize("entry,data,msg", [
    ({"dtype": "F32", "shape": [2], "data_offsets": [0, 16]}, b"\0" * 8, "outside the 8 data bytes"),
    ({"dtype": "F32", "shape": [3], "data_offsets": [0, 8]}, b"\0" * 8, "8 bytes for 3 F32 elements"),
    ({"dtype": "F32", "shape": [2], "data_offsets": [8, 0]}, b"\0" * 8, "data_offsets"),
    ({"dtype": "F32", "shape": [-2], "data_offsets": [0, 8]}, b"\0" * 8, "non-negative integers"),
    ({"dtype": "F32", "shape": [2]}, b"\0" * 8, "malformed entry"),
    ({"dtype": 7, "shape": [2], "data_offsets": [0, 8]}, b"\0" * 8, "malformed entry"),
])
def test_malformed_entries(tmp_path, entry, data, msg):
    _raw_shard(tmp_path, {"t": entry}, data)
    with pytest.raises(CheckpointError, match=msg):
        Checkpoint(str(tmp_path))


def test_load_rows_checks_before_any_copy(tmp_path):
    """Missing names, wrong shapes, a wrong destination size and unsupported dtypes
    are reported before anything is staged (no GPU is touched: CPU tensors here
    only provide a pointer that is never dereferenced)."""
    _shard(tmp_path, "m.safetensors",
           {"w": S.bf16(np.zeros(12, np.uint16), (3, 4)), "v": S.bf16(np.zeros(4, np.uint16), (4,)),
            "i": ("I32", (4,), np.zeros(4, "<i4").tobytes())})
    dst = torch.empty(16, dtype=torch.bfloat16)
    with Checkpoint(str(tmp_path)) as ck:
        with pytest.raises(CheckpointError, match="missing tensor q"):
            ck.load_rows([("q", 3)], 4, dst)
        with pytest.raises(ShapeError, match=r"w: shape \[3, 4\], expected \[4, 4\]"):
            ck.load_rows([("w", 4)], 4, dst)
        with pytest.raises(ShapeError, match=r"v: shape \[4\], expected \[1, 4\]"):
            ck.load_rows([("v", 1)], 4, dst)
        with pytest.raises(ShapeError, match="the parts hold 16 elements, dst holds 12"):
            ck.load_rows([("w", 3), ("v", 0)], 4, dst[:12])
        with pytest.raises(CheckpointError, match="unsupported dtype I32"):
            ck.load_rows([("i", 0)], 4, dst[:4])
        with pytest.raises(ShapeError, match="needs the bad counter"):
            ck.load_rows([("w", 3), ("v", 0)], 4, torch.empty(16, dtype=torch.float16))


def test_header_escapes_and_whitespace(tmp_path):
    header = ('{ "__metadata__" : {"k": "v\\"q"},\n\t"x\\u0041\\ud83d\\ude00" : '
              '{"dtype":"F16","shape":[2],"data_offsets":[0,4]} }   ').encode()
    (tmp_path / "e.safetensors").write_bytes(struct.pack("<Q", len(header)) + header + b"\0" * 4)
    with Checkpoint(str(tmp_path)) as ck:
        assert len(ck) == 1
        assert ck.info("xA\U0001F600") == ("F16", (2,))
