"""Generate the SE12 golden fixtures by running the reference codec itself.

Usage (in a container where the reference source tree is present):

    python tests/golden/make_golden.py /path/to/reference/src

For every recipe in ``cases.py`` this runs the reference's
``lws.domain.se12.codec.encode_tensor`` / ``decode_tensor``,
``lws.domain.se12.summary.se12_tensor_byte_size`` and
``lws.adapters.cuda.gemv.fallback_offsets`` (imported behind an empty
``cupy`` stub, since only its numpy host helper is used), and writes

* ``golden.json``: per case the input digest, codebook, byte size, fallback
  count and the sha256 of every stream and of the decoded bits;
* ``golden_small.npz``: the full streams of the cases small enough to commit.

The fixtures are committed; the tests only read them.
"""

from __future__ import annotations

import hashlib
import json
import pathlib
import sys
import types

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
SMALL_CASE_BYTES = 96 * 1024


def digest(array: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(array).tobytes()).hexdigest()


def main(reference_src: str) -> None:
    sys.path.insert(0, reference_src)
    sys.path.insert(0, str(HERE))
    sys.modules.setdefault("cupy", types.ModuleType("cupy"))
    from lws.adapters.cuda.gemv import fallback_offsets
    from lws.domain.se12.codec import decode_tensor, encode_tensor, fallback_tile_count
    from lws.domain.se12.summary import se12_tensor_byte_size
    from lws.domain.se12.tile import MatrixShape
    from lws.domain.weights import Bf16Weights

    import cases as recipes

    table = {}
    small = {}
    for name, (bits, rows, cols) in recipes.all_cases().items():
        pattern = np.ascontiguousarray(bits, dtype=np.uint16).view(np.int16)
        encoded = encode_tensor(Bf16Weights(bit_pattern=pattern), MatrixShape(rows=rows, cols=cols))
        decoded = decode_tensor(encoded)
        assert np.array_equal(decoded.bit_pattern, pattern), name
        streams = encoded.streams
        arrays = {
            "sm": streams.primary.sm.value,
            "ec": streams.primary.ec.value,
            "esc": streams.escape_handling.esc.value,
            "fallback_bitmap": streams.escape_handling.fallback.bitmap.value,
            "fallback_raw": streams.escape_handling.fallback.raw.value,
        }
        tile_count = (-(-rows // 16)) * (-(-cols // 256))
        offsets = fallback_offsets(arrays["fallback_bitmap"], tile_count)
        entry = {
            "rows": rows,
            "cols": cols,
            "input_sha256": digest(pattern),
            "codebook": [int(v) for v in encoded.metadata.codebook.exponents],
            "byte_size": int(se12_tensor_byte_size(encoded).value),
            "fallback_tiles": int(fallback_tile_count(encoded).value),
            "decoded_sha256": digest(decoded.bit_pattern),
            "fallback_offsets_sha256": digest(offsets),
            "streams": {k: {"sha256": digest(v), "dtype": str(v.dtype), "shape": list(v.shape)} for k, v in arrays.items()},
        }
        total = sum(v.nbytes for v in arrays.values())
        entry["stored_in_npz"] = total <= SMALL_CASE_BYTES
        if entry["stored_in_npz"]:
            for key, value in arrays.items():
                small[f"{name}/{key}"] = value
            small[f"{name}/fallback_offsets"] = offsets
        table[name] = entry
        print(f"{name:36s} {rows}x{cols} bytes={entry['byte_size']} fallback={entry['fallback_tiles']} npz={entry['stored_in_npz']}")

    (HERE / "golden.json").write_text(json.dumps(table, indent=1, sort_keys=True) + "\n")
    np.savez_compressed(HERE / "golden_small.npz", **small)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit(f"usage: python {pathlib.Path(__file__).name} <path to the reference's src directory (holds lws/)>")
    main(sys.argv[1])
