"""SE12 weight offload: decoder layers that do not fit the VRAM budget stay in
pinned host memory and are streamed to the GPU on every token, double
buffered, while the previous layer computes with the same kernels as a
resident layer (the reference's weight-offload feature,
.spec/features/weight-offload/spec.md US-016 / AC-029..AC-030 and design.md
"Pipeline", which the reference specifies but has not built).

* ``place_layers``: the pure placement rule. Walk the layers in forward
  order and keep them resident while they fit the budget minus two staging
  buffers sized for the largest layer; stream the rest. The same rule for
  both formats, so SE12 and BF16 differ only in bytes.
* ``LayerStreamer``: one contiguous pinned host block per streamed layer
  (every stream 256-byte aligned, SE12 derived tables included, so a staged
  layer needs no preparation), two device staging buffers, a copy stream
  and events. Streamed layers are used in a fixed cycle, token after
  token; the p-th use goes to staging slot p % 2. ``acquire`` makes the
  current stream wait for the layer's copy, ``release`` records that the
  layer's kernels are queued and lets the copy stream refill the slot with
  the layer two uses later (wrapping to the next token's first layers, so
  copies run continuously across tokens).
* ``offload_model``: applies this to a model compressed by
  ``runtime.compress_model``: the decoder layers past the budget get
  forward hooks that acquire and release their layer, and their compressed
  layers compute from the staging buffers.

Both formats stream through the same pipeline: SE12 matrices
(``DeviceSe12Matrix``, segmented ones included) or dense BF16 weights.
"""

from __future__ import annotations

import dataclasses
from typing import Sequence

import torch

from .device import DeviceSe12Matrix

ALIGN = 256


def _round(n: int) -> int:
    return (n + ALIGN - 1) // ALIGN * ALIGN


# ------------------------------------------------------------------ placement


@dataclasses.dataclass(frozen=True)
class Placement:
    resident: tuple
    streamed: tuple
    resident_bytes: int
    streamed_bytes: int
    staging_bytes: int


def place_layers(layer_bytes: Sequence[int], budget_bytes: int) -> Placement:
    """Which layers stay resident under ``budget_bytes`` of VRAM for layer
    weights (design.md "Pipeline": forward order; the budget pays for two
    staging buffers as soon as anything is streamed)."""
    sizes = [int(b) for b in layer_bytes]
    if any(b < 0 for b in sizes) or budget_bytes < 0:
        raise ValueError("sizes and budget must be non-negative")
    if sum(sizes) <= budget_bytes:
        return Placement(tuple(range(len(sizes))), (), sum(sizes), 0, 0)
    staging = 2 * max(sizes)
    room = budget_bytes - staging
    resident, used = [], 0
    for i, b in enumerate(sizes):
        if used + b > room:
            break
        resident.append(i)
        used += b
    streamed = tuple(range(len(resident), len(sizes)))
    return Placement(tuple(resident), streamed, used, sum(sizes[i] for i in streamed), staging)


def predicted_stream_ratio(bf16_bytes: float, se12_bytes: float, resident_bytes: float) -> float:
    """Streamed SE12 bytes over streamed BF16 bytes when both formats keep
    ``resident_bytes`` of weights in VRAM (design.md: (r T - R) / (T - R),
    0 once SE12 fits)."""
    if bf16_bytes <= resident_bytes:
        raise ValueError("BF16 fits: nothing is streamed")
    return max(0.0, se12_bytes - resident_bytes) / (bf16_bytes - resident_bytes)


# ------------------------------------------------------------------ host blocks


_SE12_FIELDS = ("sm", "ec", "esc", "fallback_bitmap", "fallback_raw", "escape_pos", "fallback_index")


def _byte_view(t: torch.Tensor) -> torch.Tensor:
    return t.contiguous().reshape(-1).view(torch.uint8)


@dataclasses.dataclass
class _Entry:
    """One matrix of a layer block: where each of its tensors lies."""
    kind: str                  # "se12" or "bf16"
    meta: dict                 # shape, codebook / segments, fallback tiles
    offsets: dict              # field -> (offset, bytes, dtype)


def _layout(layer) -> tuple:
    entries, off = [], 0
    for m in layer:
        fields = {}
        if isinstance(m, DeviceSe12Matrix):
            raw_bytes = m.fallback_tiles * 4096 * 2
            for name in _SE12_FIELDS:
                t = getattr(m, name)
                n = raw_bytes if name == "fallback_raw" else t.numel() * t.element_size()
                fields[name] = (off, n, t.dtype)
                off = _round(off + max(n, 16))
            meta = {"rows": m.rows, "cols": m.cols, "segments": m.segments, "fallback_tiles": m.fallback_tiles}
            entries.append(_Entry("se12", meta, fields))
        else:
            w = m
            if w.dtype != torch.bfloat16 or w.dim() != 2:
                raise TypeError("dense layers stream BF16 [rows, cols] weights")
            n = w.numel() * 2
            fields["weight"] = (off, n, torch.bfloat16)
            off = _round(off + n)
            entries.append(_Entry("bf16", {"rows": w.shape[0], "cols": w.shape[1]}, fields))
    return entries, off


def _fill_block(layer, entries, block: torch.Tensor) -> None:
    for m, e in zip(layer, entries):
        if e.kind == "se12":
            for name in _SE12_FIELDS:
                off, n, _ = e.offsets[name]
                if n:
                    block[off:off + n].copy_(_byte_view(getattr(m, name))[:n])
        else:
            off, n, _ = e.offsets["weight"]
            block[off:off + n].copy_(_byte_view(m))


def _views(entries, buf: torch.Tensor) -> list:
    """Per matrix: a DeviceSe12Matrix over the staging buffer (derived
    tables included, no preparation) or a BF16 weight view."""
    out = []
    for e in entries:
        def field(name, _e=e):
            off, n, dtype = _e.offsets[name]
            return buf[off:off + n].view(dtype)
        if e.kind == "bf16":
            out.append(field("weight").view(e.meta["rows"], e.meta["cols"]))
            continue
        meta = e.meta
        out.append(DeviceSe12Matrix(meta["rows"], meta["cols"], meta["segments"][0][1], field("sm"), field("ec"), field("esc"),
                                    field("fallback_bitmap"), field("fallback_raw"), segments=meta["segments"],
                                    derived=(field("escape_pos"), field("fallback_index"))))
    return out


def layer_nbytes(layer) -> int:
    """Bytes a layer occupies in a block (its matrices' streams and derived
    tables, or its BF16 weights, each 256-byte aligned)."""
    return _layout(layer)[1]


# ------------------------------------------------------------------ streamer


class LayerStreamer:
    """Streams layers (lists of ``DeviceSe12Matrix`` or BF16 weight tensors)
    from pinned host memory through two device staging buffers.

    The given device copies are read once into the pinned blocks; drop them
    afterwards to free their VRAM. Use, per token, for every streamed layer
    j in order: ``views = acquire(j)``, launch the layer's kernels on the
    current stream, ``release(j)``."""

    def __init__(self, layers: Sequence[Sequence], device: torch.device | str = "cuda"):
        if not layers:
            raise ValueError("no layers to stream")
        self.device = torch.device(device)
        self.n = len(layers)
        layouts = [_layout(layer) for layer in layers]
        self.entries = [lay[0] for lay in layouts]
        self.block_bytes = [lay[1] for lay in layouts]
        self.blocks = []
        for layer, entries, nbytes in zip(layers, self.entries, self.block_bytes):
            block = torch.empty(nbytes, dtype=torch.uint8, pin_memory=True)
            _fill_block(layer, entries, block)
            self.blocks.append(block)
        torch.cuda.synchronize(self.device)
        cap = max(self.block_bytes)
        self.staging = [torch.empty(cap, dtype=torch.uint8, device=self.device) for _ in range(2)]
        # views[slot][j]: layer j's matrices as they lie in staging slot `slot`
        self.views = [[_views(entries, buf) for entries in self.entries] for buf in self.staging]
        self.copy_stream = torch.cuda.Stream(self.device)
        self.copied = [torch.cuda.Event() for _ in range(2)]
        self.consumed = [torch.cuda.Event() for _ in range(2)]
        self._position = 0       # position (token * n + j) of the next acquire
        self._issued = 0         # positions whose copies are issued
        self._slot_of: dict = {}

    @property
    def streamed_bytes(self) -> int:
        """Bytes copied per token."""
        return sum(self.block_bytes)

    def _issue(self) -> None:
        p = self._issued
        slot, j = p % 2, p % self.n
        with torch.cuda.stream(self.copy_stream):
            if p >= 2:
                self.copy_stream.wait_event(self.consumed[slot])
            nbytes = self.block_bytes[j]
            self.staging[slot][:nbytes].copy_(self.blocks[j], non_blocking=True)
            self.copied[slot].record(self.copy_stream)
        self._issued += 1

    def acquire(self, j: int) -> list:
        """Waits (on the current stream) for streamed layer j and returns its
        matrices in the staging buffer. Layers must be acquired in order."""
        if j != self._position % self.n:
            raise RuntimeError(f"layer {j} acquired out of order (expected {self._position % self.n})")
        # this position and the next: their slots' previous layers are released
        while self._issued < self._position + 2:
            self._issue()
        slot = self._position % 2
        torch.cuda.current_stream(self.device).wait_event(self.copied[slot])
        return self.views[slot][j]

    def release(self, j: int) -> None:
        """Marks layer j's kernels as queued on the current stream; its slot
        is refilled once they have run."""
        slot = self._position % 2
        self.consumed[slot].record(torch.cuda.current_stream(self.device))
        self._position += 1
        while self._issued < self._position + 2:
            self._issue()

    def synchronize(self) -> None:
        torch.cuda.current_stream(self.device).wait_stream(self.copy_stream)


# ------------------------------------------------------------------ models


def _layer_matrices(layer: torch.nn.Module):
    """The compressed layers of a decoder layer and the distinct matrices
    they compute from (a projection group's matrix once)."""
    from .runtime import CompressedLinear

    mods = [m for m in layer.modules() if isinstance(m, CompressedLinear)]
    mats = []
    for m in mods:
        if all(m.matrix is not x for x in mats):
            mats.append(m.matrix)
    return mods, mats


def offload_model(model: torch.nn.Module, budget_bytes: int, layers_attr: str = "model.layers",
                  device: torch.device | str = "cuda") -> Placement:
    """Streams the decoder layers of a compressed model (``compress_model``
    or ``load_packed``) that do not fit ``budget_bytes``: their matrices move
    to pinned host memory and forward hooks acquire / release them around
    each layer. Embeddings, the LM head and everything outside the decoder
    layers stay resident. Returns the placement."""
    layers = model.get_submodule(layers_attr)
    per_layer = [_layer_matrices(layer) for layer in layers]
    placement = place_layers([layer_nbytes(mats) for _, mats in per_layer], budget_bytes)
    if not placement.streamed:
        return placement
    streamer = LayerStreamer([per_layer[i][1] for i in placement.streamed], device)

    for j, i in enumerate(placement.streamed):
        mods, mats = per_layer[i]
        # each compressed layer's matrix, as an index into the layer's list
        index = [next(k for k, x in enumerate(mats) if x is m.matrix) for m in mods]

        def point_to(views, _mods=mods, _index=index):
            for m, k in zip(_mods, _index):
                m.matrix = views[k]
                if m.group is not None:
                    m.group.matrix = views[k]

        # drop the resident copies now: the layer computes from staging only
        point_to(streamer.views[j % 2][j])

        def pre_hook(module, args, _j=j, _point_to=point_to):
            _point_to(streamer.acquire(_j))

        def post_hook(module, args, output, _j=j):
            streamer.release(_j)

        layers[i].register_forward_pre_hook(pre_hook)
        layers[i].register_forward_hook(post_hook)
    del per_layer
    model._se12_streamer = streamer
    torch.cuda.empty_cache()
    return placement


__all__ = ["LayerStreamer", "Placement", "layer_nbytes", "offload_model", "place_layers", "predicted_stream_ratio"]
