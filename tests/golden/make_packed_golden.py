"""Golden packed file: run the reference packer (``lws.pack``) on a small model.

Usage (where the reference source tree is present):

    python tests/golden/make_packed_golden.py /path/to/reference/src

Writes ``golden_pack.json``: the sha256 of the packed shard that the
reference's ``pack_model`` + ``SafetensorsPackedStore`` produce for the model
of ``packed_model_tensors()`` (BF16 2-D tensors with concentrated, padded and
forced-fallback content, a 1-D BF16 bias, an fp32 scale and a bool mask), and
its summary counts. The tests rebuild the same model and hold this package's
writer and GPU packer to that hash.
"""

from __future__ import annotations

import hashlib
import json
import pathlib
import sys
import tempfile

import numpy as np
import torch

HERE = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))

import cases  # noqa: E402

SHARD = "model-00001-of-00001.safetensors"


def _bf16(bits, rows, cols) -> torch.Tensor:
    return torch.from_numpy(np.asarray(bits, dtype=np.uint16).view(np.int16).reshape(rows, cols).copy()).view(torch.bfloat16)


def packed_model_tensors() -> dict:
    """The small model packed for the golden (deterministic)."""
    t = {}
    t["layer0.weight"] = _bf16(*cases.concentrated(64, 512, 1, 120, 135))
    t["layer1.weight"] = _bf16(*cases.concentrated(32, 256, 2, 120, 135))
    t["embed.weight"] = _bf16(*cases.synthetic_weights(48, 300, seed=6))
    bits, rows, cols = cases.forced_fallback_tile()
    t["fallback.weight"] = _bf16(bits, rows, cols)
    t["layer.bias"] = (torch.arange(64, dtype=torch.float32) / 64.0).to(torch.bfloat16)
    t["norm.scale"] = torch.linspace(0.0, 1.0, 64, dtype=torch.float32)
    t["mask"] = torch.zeros(10, dtype=torch.bool)
    return t


def write_model(model_dir: pathlib.Path) -> None:
    import safetensors.torch

    model_dir.mkdir(parents=True, exist_ok=True)
    safetensors.torch.save_file(packed_model_tensors(), str(model_dir / SHARD))


def main(reference_src: str) -> None:
    sys.path.insert(0, reference_src)
    from lws.adapters.safetensors.packed_store import SafetensorsPackedStore
    from lws.adapters.safetensors.weight_source import SafetensorsWeightSource
    from lws.application.codec.pack_model import pack_model

    with tempfile.TemporaryDirectory() as tmp:
        model_dir, out_dir = pathlib.Path(tmp) / "model", pathlib.Path(tmp) / "packed"
        write_model(model_dir)
        summary = pack_model(SafetensorsWeightSource(model_dir), SafetensorsPackedStore(out_dir))
        data = (out_dir / SHARD).read_bytes()
    record = {
        "shard": SHARD,
        "sha256": hashlib.sha256(data).hexdigest(),
        "bytes": len(data),
        "encoded": summary.tensor_counts.encoded.value,
        "passed_through": summary.tensor_counts.passed_through.value,
        "original_bytes": summary.eligible_sizes.original.value,
        "packed_bytes": summary.eligible_sizes.packed.value,
        "generator": "reference lws.application.codec.pack_model + SafetensorsPackedStore",
    }
    (HERE / "golden_pack.json").write_text(json.dumps(record, indent=1) + "\n")
    print(json.dumps(record))


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit(f"usage: python {pathlib.Path(__file__).name} <path to the reference's src directory (holds lws/)>")
    main(sys.argv[1])
