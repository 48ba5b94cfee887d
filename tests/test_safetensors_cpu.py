"""aex_safetensors_scan on CPU (no GPU needed): shard discovery (single file,
directory with model.safetensors.index.json, directory without it, later shard
overriding an earlier one, as SafetensorsLoader.shardFileNames /
loadMergedArrays, Sources/ImarelloWeights/SafetensorsLoader.swift:6-29 and
SafetensorsLoader+MLX.swift:6-16) and rejection of malformed files."""
import json
import struct

import pytest
import torch
from safetensors.torch import save_file

from aestrix_b200 import _lib, dit


def _tensors(seed):
    g = torch.Generator().manual_seed(seed)
    return {
        "blk.lin.weight": torch.randint(0, 2**31, (4, 8), generator=g, dtype=torch.int64).to(torch.uint32),
        "blk.lin.scales": torch.rand(4, 1, generator=g).to(torch.bfloat16),
        "blk.lin.biases": torch.rand(4, 1, generator=g).to(torch.bfloat16),
        "blk.norm.weight": torch.rand(128, generator=g),
    }


def _header(path):
    raw = open(path, "rb").read()
    n = struct.unpack("<Q", raw[:8])[0]
    return json.loads(raw[8:8 + n]), 8 + n


def test_scan_single_file_matches_header(tmp_path):
    f = tmp_path / "m.safetensors"
    save_file(_tensors(1), str(f))
    got = dit.scan_safetensors(f)
    hdr, base = _header(f)
    hdr.pop("__metadata__", None)
    assert set(got) == set(hdr)
    for k, v in hdr.items():
        dtype, shape, off, nb = got[k]
        assert dtype == v["dtype"] and list(shape) == v["shape"]
        assert off == base + v["data_offsets"][0] and nb == v["data_offsets"][1] - v["data_offsets"][0]


def test_scan_directory_with_and_without_index(tmp_path):
    a, b = _tensors(1), _tensors(2)
    b = {"other." + k: v for k, v in b.items()}
    save_file(a, str(tmp_path / "model-00001-of-00002.safetensors"))
    save_file(b, str(tmp_path / "model-00002-of-00002.safetensors"))
    save_file({"stray.weight": torch.zeros(128)}, str(tmp_path / "zz-not-in-index.safetensors"))
    wm = {k: "model-00001-of-00002.safetensors" for k in a}
    wm.update({k: "model-00002-of-00002.safetensors" for k in b})
    (tmp_path / "model.safetensors.index.json").write_text(json.dumps({"metadata": {}, "weight_map": wm}))
    got = dit.scan_safetensors(tmp_path)
    assert set(got) == set(a) | set(b)  # the index names the shards: the stray file is not read
    (tmp_path / "model.safetensors.index.json").unlink()
    assert set(dit.scan_safetensors(tmp_path)) == set(a) | set(b) | {"stray.weight"}


def test_later_shard_overrides(tmp_path):
    save_file({"x.weight": torch.zeros(128)}, str(tmp_path / "a.safetensors"))
    save_file({"x.weight": torch.zeros(128, dtype=torch.bfloat16)}, str(tmp_path / "b.safetensors"))
    assert dit.scan_safetensors(tmp_path)["x.weight"][0] == "BF16"


@pytest.mark.parametrize("case", ["missing", "short", "hlen", "json", "offsets", "dtype", "empty_dir"])
def test_scan_rejects_malformed(tmp_path, case):
    f = tmp_path / "bad.safetensors"
    good = tmp_path / "good.safetensors"
    save_file({"t.weight": torch.zeros(128)}, str(good))
    raw = good.read_bytes()
    n = struct.unpack("<Q", raw[:8])[0]
    hdr = json.loads(raw[8:8 + n])
    if case == "missing":
        f = tmp_path / "nope.safetensors"
    elif case == "short":
        f.write_bytes(raw[:5])
    elif case == "hlen":
        f.write_bytes(struct.pack("<Q", len(raw)) + raw[8:])
    elif case == "json":
        f.write_bytes(struct.pack("<Q", n) + b"{" * n + raw[8 + n:])
    elif case in ("offsets", "dtype"):
        if case == "offsets":
            hdr["t.weight"]["data_offsets"][1] += 4
        else:
            hdr["t.weight"]["dtype"] = "Q99"
        h = json.dumps(hdr).encode()
        f.write_bytes(struct.pack("<Q", len(h)) + h + raw[8 + n:])
    elif case == "empty_dir":
        f = tmp_path / "empty"
        f.mkdir()
    with pytest.raises(_lib.AexError) as e:
        dit.scan_safetensors(f)
    assert e.value.code == _lib.AEX_ERR_INVALID_ARG
