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
    - ``"by_rows"`` (the default): a fixed rule on the input's row count,
      fused for decode-sized inputs (at most ``FUSED_MAX_ROWS`` rows), exact
      for prefill (AC-025's dispatch rule). The rule depends on the shape
      only: there is no run-time choice and no dense fallback of the fused
      path, which stays the product's only GEMV.
* ``CompressedEmbedding`` replaces an ``nn.Embedding``: a lookup decodes
  only the requested rows (row-tile decode); as a tied LM head it serves
  through the GEMV path (``as_linear``).
* ``compress_model(model)`` swaps every eligible layer of a live model;
  ``load_packed(packed_dir, model)`` fills a model skeleton from a packed
  directory written by ``lws.pack`` or ``se12_b200.packed.pack_model``.
  With ``group=True`` (the default) the projections of one block that read
  the same input (q/k/v, gate/up) share one segmented matrix: the first of
  them to run computes all of their outputs in one fused GEMV and the
  others take their rows of it.

No CPU path: every compressed layer needs the CUDA library.
"""

from __future__ import annotations

import pathlib

import torch
import torch.nn.functional as F

from .device import DeviceSe12Matrix

FUSED_MAX_ROWS = 16
MODES = ("exact", "fused", "by_rows")


def _check_mode(mode: str) -> str:
    if mode not in MODES:
        raise ValueError(f"mode must be one of {MODES}, got {mode!r}")
    return mode


class ProjectionGroup:
    """Projections that multiply the same input, held as one segmented
    matrix (``DeviceSe12Matrix.concatenate`` of their own matrices).

    ``output(member, x)`` returns the whole group's fused GEMV of x. The
    result of a call is kept for the other members: each of them takes it
    once, for the same input; any other call computes afresh. So a block
    that runs q_proj, k_proj and v_proj on one hidden state (also while a
    CUDA graph captures it) runs one GEMV.

    "The same input" is checked against the tensor the result was computed
    from, which the group holds a reference to until every other member has
    taken the result: its storage stays allocated, so no other tensor can
    appear at its address in the meantime, and an in-place write to it bumps
    its version. A member whose input has another storage offset, shape,
    dtype, version or stream computes afresh."""

    def __init__(self, matrix: DeviceSe12Matrix, members: tuple):
        self.matrix = matrix
        self.members = tuple(members)
        self._x = None        # the input of the kept result (kept alive while members are pending)
        self._key = None
        self._y = None
        self._pending: set = set()

    @staticmethod
    def _key_of(x: torch.Tensor):
        stream = torch.cuda.current_stream(x.device).cuda_stream if x.is_cuda else None
        return (x.untyped_storage().data_ptr(), x.storage_offset(), tuple(x.stride()), x._version, tuple(x.shape),
                x.dtype, stream)

    def output(self, member: str, x: torch.Tensor) -> torch.Tensor:
        if member in self._pending and self._x is not None and self._key_of(x) == self._key:
            self._pending.discard(member)
            y = self._y
            if not self._pending:
                self._x = self._y = self._key = None
            return y
        y = self.matrix.gemv(x)
        self._pending = set(self.members) - {member}
        if self._pending:
            self._x, self._key, self._y = x, self._key_of(x), y
        else:
            self._x = self._y = self._key = None
        return y


class CompressedLinear(torch.nn.Module):
    """``nn.Linear`` whose weight lives on the GPU as SE12 streams only.

    With ``group`` the weight is rows ``rows`` of the group's segmented
    matrix (its own segment): the fused path takes its slice of the group's
    GEMV, the exact path decodes just those rows."""

    def __init__(self, matrix: DeviceSe12Matrix, bias: torch.Tensor | None = None, mode: str = "by_rows",
                 group: ProjectionGroup | None = None, member: str | None = None, rows: tuple | None = None):
        super().__init__()
        self.matrix = matrix
        self.group, self.member = group, member
        self.row_range = tuple(rows) if rows is not None else (0, matrix.rows)
        self.in_features, self.out_features = matrix.cols, self.row_range[1] - self.row_range[0]
        self.mode = _check_mode(mode)
        self._row_ids = None
        if bias is not None:
            self.register_buffer("bias", bias.detach().to(matrix.device))
        else:
            self.bias = None

    @classmethod
    def from_linear(cls, linear: torch.nn.Linear, mode: str = "by_rows", device="cuda") -> "CompressedLinear":
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
        if self.group is None:
            return self.matrix.decode()
        if self._row_ids is None:
            self._row_ids = torch.arange(*self.row_range, dtype=torch.int32, device=self.matrix.device)
        return self.matrix.decode_rows(self._row_ids)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        rows = x.numel() // self.in_features if self.in_features else 0
        if self.mode == "exact" or (self.mode == "by_rows" and rows > FUSED_MAX_ROWS):
            w = self.weight_bf16()
            return F.linear(x, w if x.dtype == torch.bfloat16 else w.to(x.dtype), self.bias)
        lead = x.shape[:-1]
        x2 = x.reshape(-1, self.in_features)
        if self.group is None:
            y = self.matrix.gemv(x2)
        else:
            y = self.group.output(self.member, x2)[:, self.row_range[0]:self.row_range[1]]
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

    def as_linear(self, mode: str = "by_rows") -> CompressedLinear:
        """The tied output projection over the same streams (the LM head)."""
        return CompressedLinear(self.matrix, None, mode)


def _embed_scale(emb: torch.nn.Embedding) -> torch.Tensor | None:
    scale = getattr(emb, "embed_scale", None)
    return scale if isinstance(scale, torch.Tensor) else None


def _set_module(model: torch.nn.Module, name: str, module: torch.nn.Module) -> None:
    parent_name, _, child = name.rpartition(".")
    parent = model.get_submodule(parent_name) if parent_name else model
    setattr(parent, child, module)


# Sibling projections that read the same input: (member names), grouped
# when a module has all of them as BF16 linears with one in_features.
GROUPABLE = (("q_proj", "k_proj", "v_proj"), ("gate_proj", "up_proj"))


def group_projections(model: torch.nn.Module) -> int:
    """Replaces each set of sibling ``CompressedLinear`` projections that
    read the same input (``GROUPABLE``) by members of one
    ``ProjectionGroup``; their separate matrices are released. Returns the
    number of groups made."""
    made = 0
    for parent_name, parent in list(model.named_modules()):
        for names in GROUPABLE:
            mods = [getattr(parent, n, None) for n in names]
            if not all(isinstance(m, CompressedLinear) and m.group is None for m in mods):
                continue
            mats = [m.matrix for m in mods]
            if len({id(m) for m in mats}) != len(mats) or len({m.cols for m in mats}) != 1:
                continue
            if any(m.rows % 16 for m in mats[:-1]) or sum(len(m.segments) for m in mats) > 4:
                continue
            group = ProjectionGroup(DeviceSe12Matrix.concatenate(mats), names)
            r0 = 0
            for n, m in zip(names, mods):
                r1 = r0 + m.out_features
                setattr(parent, n, CompressedLinear(group.matrix, m.bias, m.mode, group=group, member=n, rows=(r0, r1)))
                r0 = r1
            made += 1
    return made


def compress_model(model: torch.nn.Module, mode: str = "by_rows", device="cuda", embeddings: bool = True,
                   group: bool = True) -> torch.nn.Module:
    """Replaces every BF16 ``nn.Linear`` (and, with ``embeddings``, every BF16
    ``nn.Embedding``) of ``model`` in place. Layers that share one weight
    tensor (a tied embedding and LM head) share one set of streams. With
    ``group``, sibling projections that read the same input share one
    segmented matrix (``group_projections``)."""
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
    model = model.to(device)
    if group:
        group_projections(model)
    return model


def load_packed(packed_dir: str | pathlib.Path, model: torch.nn.Module, mode: str = "by_rows", device="cuda",
                group: bool = True) -> torch.nn.Module:
    """Fills ``model`` from a packed directory: each ``nn.Linear`` /
    ``nn.Embedding`` whose ``<name>.weight`` is an SE12 entry becomes a
    compressed layer over those streams (no BF16 copy of the weight stays on
    the GPU); every other parameter or buffer found in the file is loaded
    as is. A Linear whose weight is tied to a packed embedding (and absent
    from the file, as transformers saves tied weights once) shares that
    embedding's streams. ``model`` must be materialised (CPU or GPU, any
    initial values): its own buffers computed at construction, such as
    rotary tables, are kept. ``group`` as for ``compress_model``."""
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
    if group:
        group_projections(model)
    return model


__all__ = ["CompressedEmbedding", "CompressedLinear", "FUSED_MAX_ROWS", "GROUPABLE", "ProjectionGroup", "compress_model",
           "group_projections", "load_packed"]
