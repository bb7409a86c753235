"""Drop-in compressed layers for PyTorch models (the ``lws.runtime`` slice of
the model-integration feature: .spec/features/model-integration/spec.md
US-008/US-014, tasks.md T-007, which the reference specifies but has not
built).

* ``CompressedLinear`` replaces an ``nn.Linear`` and keeps only the SE12
  streams of its weight on the GPU. Modes:
    - ``"exact"``: decode the weight (bit-exact) and run the same
      ``F.linear`` as the original layer, so outputs are identical bit for
      bit to the uncompressed model (AC-016);
    - ``"fused"``: the fused decode + GEMV kernel, fp32 accumulation, output
      cast to the activation dtype (chunks of 16 rows for larger batches);
    - ``"auto"``: fused for decode-sized inputs (at most ``FUSED_MAX_ROWS``
      rows), exact for prefill (AC-025's dispatch rule with this GPU's
      measured path: the fused kernel is the product's only GEMV).
* ``CompressedEmbedding`` replaces an ``nn.Embedding``: a lookup decodes
  only the requested rows (row-tile decode); as a tied LM head it serves
  through the GEMV path (``as_linear``).
* ``compress_model(model)`` swaps every eligible layer of a live model;
  ``load_packed(packed_dir, model)`` fills a model skeleton from a packed
  directory written by ``lws.pack`` or ``se12_b200.packed.pack_model``.

No CPU path: every compressed layer needs the CUDA library.
"""

from __future__ import annotations

import pathlib

import torch
import torch.nn.functional as F

from .device import DeviceSe12Matrix

FUSED_MAX_ROWS = 16
MODES = ("exact", "fused", "auto")


def _check_mode(mode: str) -> str:
    if mode not in MODES:
        raise ValueError(f"mode must be one of {MODES}, got {mode!r}")
    return mode


class CompressedLinear(torch.nn.Module):
    """``nn.Linear`` whose weight lives on the GPU as SE12 streams only."""

    def __init__(self, matrix: DeviceSe12Matrix, bias: torch.Tensor | None = None, mode: str = "auto"):
        super().__init__()
        self.matrix = matrix
        self.in_features, self.out_features = matrix.cols, matrix.rows
        self.mode = _check_mode(mode)
        if bias is not None:
            self.register_buffer("bias", bias.detach().to(matrix.device))
        else:
            self.bias = None

    @classmethod
    def from_linear(cls, linear: torch.nn.Linear, mode: str = "auto", device="cuda") -> "CompressedLinear":
        from .codec import encode_device

        w = linear.weight.detach()
        if w.dtype != torch.bfloat16:
            raise TypeError(f"only BF16 weights are SE12-eligible, got {w.dtype}")
        matrix = encode_device(w.to(device))
        return cls(matrix, linear.bias, mode)

    def extra_repr(self) -> str:
        return f"in_features={self.in_features}, out_features={self.out_features}, bias={self.bias is not None}, mode={self.mode}"

    def weight_bf16(self) -> torch.Tensor:
        """The exact BF16 weight, decoded on the GPU (transient)."""
        return self.matrix.decode()

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        rows = x.numel() // self.in_features if self.in_features else 0
        if self.mode == "exact" or (self.mode == "auto" and rows > FUSED_MAX_ROWS):
            w = self.matrix.decode()
            return F.linear(x, w if x.dtype == torch.bfloat16 else w.to(x.dtype), self.bias)
        lead = x.shape[:-1]
        y = self.matrix.gemv(x.reshape(-1, self.in_features))
        if self.bias is not None:
            y = y + self.bias.float()
        return y.to(x.dtype).reshape(*lead, self.out_features)


class CompressedEmbedding(torch.nn.Module):
    """``nn.Embedding`` whose table lives on the GPU as SE12 streams only; a
    lookup decodes the requested rows exactly. ``scale`` reproduces scaled
    embeddings (a subclass that multiplies its output by an ``embed_scale``
    buffer cast to the table's dtype, as transformers' Gemma models do)."""

    def __init__(self, matrix: DeviceSe12Matrix, padding_idx: int | None = None, scale: torch.Tensor | None = None):
        super().__init__()
        self.matrix = matrix
        self.num_embeddings, self.embedding_dim = matrix.rows, matrix.cols
        self.padding_idx = padding_idx
        if scale is not None:
            self.register_buffer("embed_scale", scale.detach().to(matrix.device))
        else:
            self.embed_scale = None

    @classmethod
    def from_embedding(cls, emb: torch.nn.Embedding, device="cuda") -> "CompressedEmbedding":
        from .codec import encode_device

        w = emb.weight.detach()
        if w.dtype != torch.bfloat16:
            raise TypeError(f"only BF16 tables are SE12-eligible, got {w.dtype}")
        return cls(encode_device(w.to(device)), emb.padding_idx, _embed_scale(emb))

    def extra_repr(self) -> str:
        return f"{self.num_embeddings}, {self.embedding_dim}"

    def forward(self, ids: torch.Tensor) -> torch.Tensor:
        rows = self.matrix.decode_rows(ids.reshape(-1).to(torch.int32)).view(*ids.shape, self.embedding_dim)
        if self.embed_scale is not None:
            rows = rows * self.embed_scale.to(rows.dtype)
        return rows

    def as_linear(self, mode: str = "auto") -> CompressedLinear:
        """The tied output projection over the same streams (the LM head)."""
        return CompressedLinear(self.matrix, None, mode)


def _embed_scale(emb: torch.nn.Embedding) -> torch.Tensor | None:
    scale = getattr(emb, "embed_scale", None)
    return scale if isinstance(scale, torch.Tensor) else None


def _set_module(model: torch.nn.Module, name: str, module: torch.nn.Module) -> None:
    parent_name, _, child = name.rpartition(".")
    parent = model.get_submodule(parent_name) if parent_name else model
    setattr(parent, child, module)


def compress_model(model: torch.nn.Module, mode: str = "auto", device="cuda", embeddings: bool = True) -> torch.nn.Module:
    """Replaces every BF16 ``nn.Linear`` (and, with ``embeddings``, every BF16
    ``nn.Embedding``) of ``model`` in place. Layers that share one weight
    tensor (a tied embedding and LM head) share one set of streams."""
    _check_mode(mode)
    shared: dict = {}
    targets = [(n, m) for n, m in model.named_modules() if isinstance(m, (torch.nn.Linear, torch.nn.Embedding))]
    for name, mod in targets:
        w = mod.weight
        if w.dtype != torch.bfloat16 or (isinstance(mod, torch.nn.Embedding) and not embeddings):
            continue
        key = (w.data_ptr(), tuple(w.shape))
        if key in shared:
            matrix = shared[key]
        else:
            from .codec import encode_device

            matrix = encode_device(w.detach().to(device))
            shared[key] = matrix
        if isinstance(mod, torch.nn.Linear):
            _set_module(model, name, CompressedLinear(matrix, mod.bias, mode))
        else:
            _set_module(model, name, CompressedEmbedding(matrix, mod.padding_idx, _embed_scale(mod)))
    return model.to(device)


def load_packed(packed_dir: str | pathlib.Path, model: torch.nn.Module, mode: str = "auto", device="cuda") -> torch.nn.Module:
    """Fills ``model`` from a packed directory: each ``nn.Linear`` /
    ``nn.Embedding`` whose ``<name>.weight`` is an SE12 entry becomes a
    compressed layer over those streams (no BF16 copy of the weight stays on
    the GPU); every other parameter or buffer found in the file is loaded
    as is. A Linear whose weight is tied to a packed embedding (and absent
    from the file, as transformers saves tied weights once) shares that
    embedding's streams. ``model`` must be materialised (CPU or GPU, any
    initial values): its own buffers computed at construction, such as
    rotary tables, are kept."""
    from .format import Se12Tensor
    from .packed import read_packed

    _check_mode(mode)
    entries = read_packed(packed_dir)
    matrices: dict = {}
    by_weight: dict = {}

    def matrix_for(key: str) -> DeviceSe12Matrix:
        if key not in matrices:
            matrices[key] = DeviceSe12Matrix.from_tensor(entries[key], device)
        return matrices[key]

    layers = [(n, m) for n, m in model.named_modules() if isinstance(m, (torch.nn.Linear, torch.nn.Embedding))]
    for name, mod in layers:
        key = f"{name}.weight"
        if isinstance(entries.get(key), Se12Tensor):
            by_weight[id(mod.weight)] = key
    for name, mod in layers:
        key = f"{name}.weight"
        if not isinstance(entries.get(key), Se12Tensor):
            key = by_weight.get(id(mod.weight))  # tied to a packed weight
            if key is None:
                continue
        m = matrix_for(key)
        if isinstance(mod, torch.nn.Linear):
            bias = entries.get(f"{name}.bias") if mod.bias is not None else None
            _set_module(model, name, CompressedLinear(m, bias.to(device) if bias is not None else None, mode))
        else:
            _set_module(model, name, CompressedEmbedding(m, mod.padding_idx, _embed_scale(mod)))
    # every remaining parameter / buffer from the pass-through entries
    model = model.to(device)
    state = {k: v for k, v in entries.items() if isinstance(v, torch.Tensor)}
    own = dict(model.named_parameters())
    own.update(dict(model.named_buffers()))
    with torch.no_grad():
        for k, v in state.items():
            if k in own and own[k].shape == v.shape:
                own[k].copy_(v.to(device))
    return model


__all__ = ["CompressedEmbedding", "CompressedLinear", "FUSED_MAX_ROWS", "compress_model", "load_packed"]
