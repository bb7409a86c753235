"""Golden side tables of the reference's GPU kernel, made by running the
reference's own host helpers.

Usage (where the reference source tree is present):

    python tests/golden/make_ref_tables_golden.py /path/to/reference/src

For every recipe in ``cases.py`` this encodes with the reference's
``encode_tensor`` and runs ``lws.adapters.cuda.gemv.row_escape_offset``
(per output row and tile column, the escapes in earlier rows of the tile:
the rank the kernel starts from, src/lws/adapters/cuda/gemv.py:60-77) and
``fallback_offsets`` (gemv.py:47-57), behind an empty ``cupy`` stub, and
writes ``golden_ref_tables.json`` (shape and sha256 of each table). The
oracle's restatement (``se12_oracle.row_escape_offset``) is held to it; the
tables it makes are what the reference's kernel is given when this
repository times or tests that kernel.
"""

from __future__ import annotations

import hashlib
import json
import pathlib
import sys
import types

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent


def digest(array: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(array).tobytes()).hexdigest()


def main(reference_src: str) -> None:
    sys.path.insert(0, reference_src)
    sys.path.insert(0, str(HERE))
    sys.modules.setdefault("cupy", types.ModuleType("cupy"))
    from lws.adapters.cuda.gemv import fallback_offsets, row_escape_offset, tile_grid
    from lws.domain.se12.codec import encode_tensor
    from lws.domain.se12.tile import MatrixShape, TileShape
    from lws.domain.weights import Bf16Weights

    import cases as recipes

    tile = TileShape(rows=16, cols=256)
    table = {}
    for name, (bits, rows, cols) in recipes.all_cases().items():
        pattern = np.ascontiguousarray(bits, dtype=np.uint16).view(np.int16)
        enc = encode_tensor(Bf16Weights(bit_pattern=pattern), MatrixShape(rows=rows, cols=cols))
        tr, tc = tile_grid(rows, cols, tile)
        reo = row_escape_offset(np.asarray(enc.streams.primary.ec.value), tr * tc, tc, tile)
        fbo = fallback_offsets(np.asarray(enc.streams.escape_handling.fallback.bitmap.value), tr * tc)
        table[name] = {"rows": rows, "cols": cols, "row_escape_offset_shape": list(reo.shape),
                       "row_escape_offset": digest(reo.astype(np.int32)), "fallback_offsets": digest(fbo.astype(np.int32))}
    (HERE / "golden_ref_tables.json").write_text(json.dumps(table, indent=1, sort_keys=True) + "\n")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_ref_tables_golden.py <reference src directory>")
    main(sys.argv[1])
