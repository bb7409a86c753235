"""The packed container (lws.pack's safetensors layout): writer, GPU packer
and reader, pinned to the file the reference packer writes for the same
model (tests/golden/golden_pack.json, made by make_packed_golden.py).

Reference tests mirrored: tests/test_spec_pack.py:116-221 (byte ratio,
pass-through tensors, format metadata, unknown version refused,
determinism, end-to-end decode of the written file).
"""

from __future__ import annotations

import hashlib
import json
import pathlib

import numpy as np
import pytest
import torch

import make_packed_golden as golden_model
import se12_oracle as oracle

GOLDEN = json.loads((pathlib.Path(__file__).resolve().parent / "golden" / "golden_pack.json").read_text())


def sha(path: pathlib.Path) -> str:
    return hashlib.sha256(path.read_bytes()).hexdigest()


def source_entries(model_dir: pathlib.Path):
    """(name, tensor) in the order the reference packer reads the shard."""
    import safetensors

    with safetensors.safe_open(str(model_dir / golden_model.SHARD), framework="pt") as shard:
        return [(name, shard.get_tensor(name)) for name in shard.keys()]


def oracle_packed_entries(model_dir: pathlib.Path):
    from se12_b200.format import make_tensor

    out = []
    for name, t in source_entries(model_dir):
        if t.dtype == torch.bfloat16 and t.dim() == 2:
            bits = t.reshape(-1).view(torch.int16).numpy().view(np.uint16)
            s = oracle.encode(bits, t.shape[0], t.shape[1])
            out.append((name, make_tensor(s.rows, s.cols, s.codebook, s.sm, s.ec, s.esc, s.fallback_bitmap, s.fallback_raw)))
        else:
            out.append((name, t))
    return out


@pytest.fixture
def model_dir(tmp_path):
    d = tmp_path / "model"
    golden_model.write_model(d)
    return d


def test_writer_is_byte_identical_to_reference_packer(model_dir, tmp_path):
    from se12_b200.packed import write_packed_shard

    out = tmp_path / "packed" / golden_model.SHARD
    write_packed_shard(out, oracle_packed_entries(model_dir))
    assert sha(out) == GOLDEN["sha256"]


def test_read_packed_round_trip(model_dir, tmp_path):
    from se12_b200.format import Se12Tensor
    from se12_b200.packed import read_packed, write_packed_shard

    entries = oracle_packed_entries(model_dir)
    write_packed_shard(tmp_path / "packed" / golden_model.SHARD, entries)
    back = read_packed(tmp_path / "packed")
    assert list(back) == [name for name, _ in entries]
    for name, value in entries:
        got = back[name]
        if isinstance(value, torch.Tensor):
            assert got.dtype == value.dtype and torch.equal(got, value)
            continue
        assert isinstance(got, Se12Tensor)
        assert (got.rows, got.cols, got.codebook) == (value.rows, value.cols, value.codebook)
        for stream in ("sm", "ec", "esc", "fallback_bitmap", "fallback_raw"):
            assert np.array_equal(getattr(got, stream), getattr(value, stream)), (name, stream)
        # the file decodes to the original bits (test_spec_pack.py:206-221)
        streams = oracle.Streams(rows=got.rows, cols=got.cols, codebook=got.codebook, sm=got.sm, ec=got.ec, esc=got.esc,
                                 fallback_bitmap=got.fallback_bitmap, fallback_raw=got.fallback_raw)
        original = dict(source_entries(model_dir))[name]
        assert np.array_equal(oracle.decode(streams).reshape(-1), original.reshape(-1).view(torch.int16).numpy().view(np.uint16))


def test_unknown_format_version_is_refused(model_dir, tmp_path):
    import safetensors
    import safetensors.torch

    from se12_b200.packed import UnsupportedFormatVersionError, read_packed, write_packed_shard

    path = tmp_path / "packed" / golden_model.SHARD
    write_packed_shard(path, oracle_packed_entries(model_dir))
    with safetensors.safe_open(str(path), framework="pt") as shard:
        tensors = {k: shard.get_tensor(k) for k in shard.keys()}
        meta = json.loads(shard.metadata()["se12"])
    meta["format_version"] = 99
    safetensors.torch.save_file(tensors, str(path), metadata={"se12": json.dumps(meta)})
    with pytest.raises(UnsupportedFormatVersionError) as err:
        read_packed(path)
    assert "99" in str(err.value) and "1" in str(err.value)


def test_plain_safetensors_is_not_a_packed_file(model_dir):
    from se12_b200.packed import read_packed

    with pytest.raises(ValueError):
        read_packed(model_dir / golden_model.SHARD)


@pytest.mark.gpu
def test_gpu_packer_is_byte_identical_to_reference_packer(model_dir, tmp_path):
    from se12_b200.packed import pack_model

    out = tmp_path / "packed"
    summary = pack_model(model_dir, out)
    assert sha(out / golden_model.SHARD) == GOLDEN["sha256"]
    assert (summary.encoded, summary.passed_through) == (GOLDEN["encoded"], GOLDEN["passed_through"])
    assert (summary.original_bytes, summary.packed_bytes) == (GOLDEN["original_bytes"], GOLDEN["packed_bytes"])
    # the source files are untouched and nothing is written beside them
    assert sorted(p.name for p in model_dir.iterdir()) == [golden_model.SHARD]


@pytest.mark.gpu
def test_loaded_packed_matrices_decode_bit_exact(model_dir, tmp_path):
    from se12_b200.device import DeviceSe12Matrix
    from se12_b200.packed import load_packed_tensors, pack_model

    pack_model(model_dir, tmp_path / "packed")
    loaded = load_packed_tensors(tmp_path / "packed", "cuda")
    for name, original in source_entries(model_dir):
        got = loaded[name]
        if original.dtype == torch.bfloat16 and original.dim() == 2:
            assert isinstance(got, DeviceSe12Matrix)
            assert torch.equal(got.decode().cpu().view(torch.int16), original.view(torch.int16))
        else:
            assert got.is_cuda and torch.equal(got.cpu(), original)
