"""Device-resident SE12 matrices and the calls into libse12_b200.

``DeviceSe12Matrix`` owns the five SE12 streams in GPU memory (torch
tensors), the two derived tables the kernels use (escape positions,
fallback ranks) and the native handle with its TMA descriptors. Every
compute method launches a kernel of libse12_b200.so on the current torch
stream; nothing here computes on the CPU.
"""

from __future__ import annotations

import ctypes
import weakref

import numpy as np
import torch

from . import _lib
from .format import CODEBOOK_SIZE, ESCAPE_BUDGET, TILE_COLS, TILE_ROWS, TILE_SIZE, Se12Tensor, as_tensor, make_tensor, tile_grid

MAX_BATCH = 16


def stream_handle(device: torch.device | None = None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


class _WorkspacePool:
    """One zeroed stream-K workspace per (device, stream), grown on demand.

    Calls on one stream run in order, and every completed GEMV leaves the
    workspace's arrival counters at zero, so all matrices on a stream can
    share one workspace.
    """

    def __init__(self):
        self._buffers: dict = {}

    def get(self, device: torch.device, stream: int, nbytes: int) -> torch.Tensor:
        key = (device.index, stream)
        buf = self._buffers.get(key)
        if buf is None or buf.numel() < nbytes:
            size = max(nbytes, 1 << 20)
            buf = torch.empty(size, dtype=torch.uint8, device=device)
            _lib.call("se12_workspace_clear", ctypes.c_void_p(buf.data_ptr()), buf.numel(), ctypes.c_void_p(stream))
            self._buffers[key] = buf
        return buf

    def clear(self):
        self._buffers.clear()

    def reset(self):
        """Zeroes every pooled workspace again (after a kernel gave up on a
        wait, its flags may not be back at zero)."""
        for (index, stream), buf in self._buffers.items():
            with torch.cuda.device(index):
                _lib.call("se12_workspace_clear", ctypes.c_void_p(buf.data_ptr()), buf.numel(), ctypes.c_void_p(stream))


WORKSPACES = _WorkspacePool()


MAX_SEGMENTS = 4


class DeviceSe12Matrix:
    """An SE12-encoded [rows, cols] BF16 matrix resident on one GPU.

    ``segments`` (optional) makes it a segmented matrix: the streams are the
    tile-major concatenation of several SE12 matrices with the same columns,
    given as ``[(rows_i, codebook_i), ...]``; ``codebook`` is then ignored.
    ``concatenate`` builds one from separate matrices.

    ``derived`` (optional): ``(escape_pos, fallback_index)`` device tensors
    that already hold this matrix's derived tables (as computed for the same
    streams by a prepared matrix); the matrix then uses them as they are
    instead of allocating and preparing its own (the offload staging buffers
    receive them with the streams).
    """

    def __init__(self, rows: int, cols: int, codebook, sm: torch.Tensor, ec: torch.Tensor, esc: torch.Tensor,
                 fallback_bitmap: torch.Tensor, fallback_raw: torch.Tensor, segments=None, derived=None):
        lib = _lib.load()
        self.rows, self.cols = int(rows), int(cols)
        if segments is None:
            segments = [(self.rows, codebook)]
        self.segments = tuple((int(r), tuple(int(v) for v in book)) for r, book in segments)
        if not 1 <= len(self.segments) <= MAX_SEGMENTS:
            raise ValueError(f"1..{MAX_SEGMENTS} segments, got {len(self.segments)}")
        if any(len(book) != CODEBOOK_SIZE for _, book in self.segments):
            raise ValueError("codebook must have 15 entries")
        self.codebook = self.segments[0][1]
        self.device = sm.device
        tr, tc = tile_grid(self.rows, self.cols)
        self.tile_rows, self.tile_cols, self.tiles = tr, tc, tr * tc
        expect = {"sm": self.tiles * TILE_SIZE, "ec": self.tiles * TILE_SIZE // 2, "esc": self.tiles * ESCAPE_BUDGET,
                  "fallback_bitmap": (self.tiles + 7) // 8}
        given = {"sm": sm, "ec": ec, "esc": esc, "fallback_bitmap": fallback_bitmap}
        for name, n in expect.items():
            if given[name].numel() != n:
                raise ValueError(f"stream {name} has {given[name].numel()} bytes, expected {n}")
        self.sm, self.ec = sm.contiguous(), ec.contiguous()
        self.esc, self.fallback_bitmap = esc.contiguous().reshape(-1), fallback_bitmap.contiguous()
        raw = fallback_raw.contiguous().reshape(-1)
        if raw.numel() % TILE_SIZE:
            raise ValueError("fallback_raw must hold whole 4096-weight tiles")
        # keep a non-empty allocation so the pointer is valid and aligned
        self.fallback_raw = raw if raw.numel() else torch.zeros(8, dtype=torch.int16, device=self.device)
        self.fallback_tiles = raw.numel() // TILE_SIZE
        if derived is None:
            self.escape_pos = torch.empty(self.tiles * ESCAPE_BUDGET, dtype=torch.int16, device=self.device)
            # padded to a multiple of 4 tiles (the GEMV copies it in 16-byte groups)
            self.fallback_index = torch.empty((self.tiles + 3) // 4 * 4, dtype=torch.int32, device=self.device)
        else:
            self.escape_pos, self.fallback_index = derived
            if (self.escape_pos.numel() != self.tiles * ESCAPE_BUDGET or self.escape_pos.dtype != torch.int16
                    or self.fallback_index.numel() != (self.tiles + 3) // 4 * 4 or self.fallback_index.dtype != torch.int32):
                raise ValueError("derived tables have the wrong size or type for this matrix")

        s = _lib.Se12StreamsStruct()
        s.rows, s.cols = self.rows, self.cols
        s.tile_rows, s.tile_cols, s.escape_budget, s.format_version = TILE_ROWS, TILE_COLS, ESCAPE_BUDGET, 1
        for i, v in enumerate(self.codebook):
            s.codebook[i] = v
        s.sm, s.ec, s.esc = self.sm.data_ptr(), self.ec.data_ptr(), self.esc.data_ptr()
        s.fallback_bitmap, s.fallback_raw = self.fallback_bitmap.data_ptr(), self.fallback_raw.data_ptr()
        s.escape_pos, s.fallback_index = self.escape_pos.data_ptr(), self.fallback_index.data_ptr()
        nseg = len(self.segments)
        seg_rows = (ctypes.c_int32 * nseg)(*[r for r, _ in self.segments])
        books = (ctypes.c_uint8 * (nseg * CODEBOOK_SIZE))(*[v for _, book in self.segments for v in book])
        handle = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            _lib.check(lib.se12_matrix_create_segmented(ctypes.byref(s), nseg, seg_rows, books, ctypes.byref(handle)),
                       "se12_matrix_create_segmented")
            self._handle = handle
            self._finalizer = weakref.finalize(self, lib.se12_matrix_destroy, handle)
            if derived is None:
                _lib.check(lib.se12_matrix_prepare(handle, ctypes.c_void_p(stream_handle(self.device))), "se12_matrix_prepare")

    # ------------------------------------------------------------------ construction
    @classmethod
    def from_tensor(cls, tensor, device="cuda") -> "DeviceSe12Matrix":
        """Uploads a host Se12Tensor (this package's or the reference's)."""
        t = as_tensor(tensor)
        dev = torch.device(device)

        def up(a, dtype):
            return torch.from_numpy(np.ascontiguousarray(a).reshape(-1).view(dtype)).to(dev, non_blocking=False)

        return cls(t.rows, t.cols, t.codebook, up(t.sm, np.uint8), up(t.ec, np.uint8), up(t.esc, np.uint8),
                   up(t.fallback_bitmap, np.uint8), up(t.fallback_raw, np.int16))

    @classmethod
    def concatenate(cls, matrices) -> "DeviceSe12Matrix":
        """One segmented matrix holding ``matrices`` (same columns, same GPU;
        every one but the last with a multiple of 16 rows) one after the
        other, so that one GEMV computes all of them: y = [y_0 | y_1 | ...].
        The streams are copied; each segment keeps its codebook and its
        bytes are the matrix's own."""
        mats = list(matrices)
        if not mats:
            raise ValueError("nothing to concatenate")
        cols, device = mats[0].cols, mats[0].device
        for i, m in enumerate(mats):
            if m.cols != cols or m.device != device:
                raise ValueError("segments need the same columns and device")
            if i + 1 < len(mats) and m.rows % TILE_ROWS:
                raise ValueError("every segment but the last needs a multiple of 16 rows")
        segments = [seg for m in mats for seg in m.segments]
        if len(segments) > MAX_SEGMENTS:
            raise ValueError(f"at most {MAX_SEGMENTS} segments")
        shifts = torch.arange(7, -1, -1, device=device, dtype=torch.uint8)
        bits = torch.cat([((m.fallback_bitmap.unsqueeze(1) >> shifts) & 1).reshape(-1)[: m.tiles] for m in mats])
        tiles = bits.numel()
        bits = torch.nn.functional.pad(bits, (0, (-tiles) % 8)).reshape(-1, 8)
        bitmap = (bits << shifts).sum(dim=1, dtype=torch.int32).to(torch.uint8)
        raw = torch.cat([m.fallback_raw[: m.fallback_tiles * TILE_SIZE] for m in mats])
        return cls(sum(m.rows for m in mats), cols, segments[0][1], torch.cat([m.sm for m in mats]),
                   torch.cat([m.ec for m in mats]), torch.cat([m.esc for m in mats]), bitmap, raw, segments=segments)

    def segment_tensors(self) -> list:
        """Host copies of the segments as separate Se12Tensors (the tensors
        ``concatenate`` was given)."""
        shifts = np.arange(7, -1, -1, dtype=np.uint8)
        bits = ((self.fallback_bitmap.cpu().numpy()[:, None] >> shifts) & 1).reshape(-1)[: self.tiles]
        sm, ec, esc = self.sm.cpu().numpy(), self.ec.cpu().numpy(), self.esc.cpu().numpy()
        raw = self.fallback_raw[: self.fallback_tiles * TILE_SIZE].cpu().numpy()
        out, t0, f0 = [], 0, 0
        for rows, book in self.segments:
            t1 = t0 + tile_grid(rows, self.cols)[0] * self.tile_cols
            seg_bits = bits[t0:t1]
            f1 = f0 + int(seg_bits.sum())
            out.append(make_tensor(rows, self.cols, book, sm[t0 * TILE_SIZE:t1 * TILE_SIZE],
                                   ec[t0 * TILE_SIZE // 2:t1 * TILE_SIZE // 2], esc[t0 * ESCAPE_BUDGET:t1 * ESCAPE_BUDGET],
                                   np.packbits(seg_bits.astype(np.uint8)), raw[f0 * TILE_SIZE:f1 * TILE_SIZE]))
            t0, f0 = t1, f1
        return out

    def to_tensor(self) -> Se12Tensor:
        """Host copy of the streams as an Se12Tensor."""
        if len(self.segments) > 1:
            raise ValueError("a segmented matrix has one codebook per segment: use segment_tensors()")
        raw = self.fallback_raw[: self.fallback_tiles * TILE_SIZE]
        return make_tensor(self.rows, self.cols, self.codebook, self.sm.cpu().numpy(), self.ec.cpu().numpy(),
                           self.esc.cpu().numpy(), self.fallback_bitmap.cpu().numpy(), raw.cpu().numpy())

    @property
    def handle(self) -> ctypes.c_void_p:
        return self._handle

    @property
    def records(self) -> torch.Tensor:
        """Per-tile records the chain kernel reads (64 bytes per tile: the
        escaped weights' positions with their exponents, fallback ranks),
        built on the device on first use."""
        if getattr(self, "_records", None) is None:
            rec = torch.empty(self.tiles * ESCAPE_BUDGET, dtype=torch.int32, device=self.device)
            with torch.cuda.device(self.device):
                _lib.call("se12_matrix_prepare_records", self._handle, ctypes.c_void_p(rec.data_ptr()),
                          ctypes.c_void_p(stream_handle(self.device)))
            self._records = rec
        return self._records

    @property
    def byte_size(self) -> int:
        """Algorithmic SE12 bytes: five streams + 15 codebook bytes."""
        # a segmented matrix counts each segment's own bitmap and codebook,
        # the bytes its separate tensor has
        bitmaps = sum((tile_grid(rows, self.cols)[0] * self.tile_cols + 7) // 8 for rows, _ in self.segments)
        return (self.sm.numel() + self.ec.numel() + self.esc.numel() + bitmaps
                + self.fallback_tiles * TILE_SIZE * 2 + CODEBOOK_SIZE * len(self.segments))

    # ------------------------------------------------------------------ compute
    def gemv(self, x: torch.Tensor, out: torch.Tensor | None = None, order_matched: bool = False) -> torch.Tensor:
        """y[B, N] = x[B, K] . W^T in fp32 (x: BF16 or fp32, [K] or [B, K]).
        ``order_matched``: in bf16_gemv's launch configuration, so that the
        result equals the dense kernel's bit for bit on matrices without
        escapes of non-zero exponent (the reference spec's AC-032)."""
        return gemv_call(self, x, out, order_matched=order_matched)

    def launch_config(self, batch: int = 1) -> dict:
        """The launch se12_gemv makes for this matrix at this batch size."""
        cfg = _lib.Se12LaunchConfigStruct()
        _lib.call("se12_gemv_launch_config", self._handle, int(batch), ctypes.byref(cfg))
        return {name: getattr(cfg, name) for name, _ in cfg._fields_}

    def decode(self, out: torch.Tensor | None = None) -> torch.Tensor:
        """The exact BF16 matrix [rows, cols] on the device."""
        if out is None:
            out = torch.empty(self.rows, self.cols, dtype=torch.bfloat16, device=self.device)
        _check_out(out, self.cols)
        with torch.cuda.device(self.device):
            _lib.call("se12_decode", self._handle, ctypes.c_void_p(out.data_ptr()), out.stride(0),
                      ctypes.c_void_p(stream_handle(self.device)))
        return out

    def decode_rows(self, rows, out: torch.Tensor | None = None) -> torch.Tensor:
        """Exact BF16 rows [len(rows), cols] in request order."""
        idx = torch.as_tensor(rows, dtype=torch.int32).reshape(-1).to(self.device)
        if out is None:
            out = torch.empty(idx.numel(), self.cols, dtype=torch.bfloat16, device=self.device)
        _check_out(out, self.cols)
        with torch.cuda.device(self.device):
            _lib.call("se12_decode_rows", self._handle, ctypes.c_void_p(idx.data_ptr()), idx.numel(),
                      ctypes.c_void_p(out.data_ptr()), out.stride(0), ctypes.c_void_p(stream_handle(self.device)))
        return out


def _check_out(out: torch.Tensor, cols: int):
    if out.dtype != torch.bfloat16 or out.dim() != 2 or out.stride(1) != 1 or out.shape[1] != cols:
        raise ValueError("out must be a BF16 [n, cols] tensor with unit column stride")


def _aligned_bf16(x: torch.Tensor, cols: int) -> torch.Tensor:
    """x as a [B, ldx] BF16 view with 16-byte aligned rows (ldx % 8 == 0)."""
    if x.dim() == 1:
        x = x.unsqueeze(0)
    if x.stride(-1) == 1 and x.stride(0) % 8 == 0 and x.stride(0) >= (cols + 7) // 8 * 8 and x.data_ptr() % 16 == 0:
        return x
    ld = (cols + 7) // 8 * 8
    buf = torch.zeros(x.shape[0], ld, dtype=torch.bfloat16, device=x.device)
    buf[:, :cols] = x
    return buf


def _split_fp32(x: torch.Tensor) -> list:
    """fp32 -> three BF16 parts whose sum is x exactly (8+8+8 significant bits)."""
    hi = x.to(torch.bfloat16)
    r1 = x - hi.float()
    mid = r1.to(torch.bfloat16)
    lo = (r1 - mid.float()).to(torch.bfloat16)
    return [hi, mid, lo]


def gemv_call(m: DeviceSe12Matrix, x: torch.Tensor, out: torch.Tensor | None = None, raw_weights: torch.Tensor | None = None,
              order_matched: bool = False) -> torch.Tensor:
    """Shared GEMV driver for the fused SE12 kernel and the dense baseline
    (``order_matched``: the SE12 kernel in the dense kernel's launch
    configuration, se12_gemv_order_matched)."""
    rows, cols = (m.rows, m.cols) if m is not None else raw_weights.shape
    device = x.device
    squeeze = x.dim() == 1
    x2 = x.reshape(1, -1) if squeeze else x
    if x2.shape[-1] != cols:
        raise ValueError(f"x has {x2.shape[-1]} columns, matrix has {cols}")
    if x2.dtype == torch.float32:
        parts = _split_fp32(x2)
        ys = [gemv_call(m, p, None, raw_weights, order_matched) for p in parts]
        y = (ys[0] + ys[1]) + ys[2]
        if out is not None:
            out.copy_(y)
            y = out
        return y.reshape(-1) if squeeze else y
    if x2.dtype != torch.bfloat16:
        raise TypeError("activations must be bfloat16 or float32")
    batch = x2.shape[0]
    if out is None:
        out = torch.empty(batch, rows, dtype=torch.float32, device=device)
    if out.dtype != torch.float32 or out.stride(-1) != 1:
        raise ValueError("out must be fp32 with unit column stride")
    out2 = out.reshape(1, -1) if out.dim() == 1 else out
    stream = stream_handle(device)
    with torch.cuda.device(device):
        for b0 in range(0, batch, MAX_BATCH):
            xb = _aligned_bf16(x2[b0 : b0 + MAX_BATCH], cols)
            yb = out2[b0 : b0 + MAX_BATCH]
            nb = xb.shape[0]
            if m is not None:
                need = _lib.load().se12_gemv_workspace_bytes(m.handle, MAX_BATCH)
                ws = WORKSPACES.get(device, stream, need)
                _lib.call("se12_gemv_order_matched" if order_matched else "se12_gemv", m.handle,
                          ctypes.c_void_p(xb.data_ptr()), nb, xb.stride(0),
                          ctypes.c_void_p(yb.data_ptr()), yb.stride(0), ctypes.c_void_p(ws.data_ptr()), ws.numel(),
                          ctypes.c_void_p(stream))
            else:
                w = raw_weights
                need = _lib.load().bf16_gemv_workspace_bytes(rows, cols, MAX_BATCH)
                ws = WORKSPACES.get(device, stream, need)
                _lib.call("bf16_gemv", ctypes.c_void_p(w.data_ptr()), rows, cols, w.stride(0),
                          ctypes.c_void_p(xb.data_ptr()), nb, xb.stride(0), ctypes.c_void_p(yb.data_ptr()), yb.stride(0),
                          ctypes.c_void_p(ws.data_ptr()), ws.numel(), ctypes.c_void_p(stream))
    return out.reshape(-1) if squeeze else out


def bf16_gemv(weights: torch.Tensor, x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """Dense BF16 GEMV baseline with the same pipeline as the fused kernel."""
    if weights.dtype != torch.bfloat16 or weights.dim() != 2 or weights.stride(1) != 1:
        raise ValueError("weights must be a BF16 [rows, cols] matrix with unit column stride")
    w = weights
    if w.stride(0) % 8 or w.data_ptr() % 16:
        ld = (w.shape[1] + 7) // 8 * 8
        buf = torch.zeros(w.shape[0], ld, dtype=torch.bfloat16, device=w.device)
        buf[:, : w.shape[1]] = w
        w = buf[:, : weights.shape[1]]
    return gemv_call(None, x, out, raw_weights=w)


STATUS_WAIT_TIMEOUT = 1


def set_wait_limit_ns(ns: int) -> None:
    """Limit of the kernels' waits on other CTAs and GPUs on the current
    device (default 2 s; a short one makes a lost peer's wait run out fast)."""
    _lib.call("se12_set_wait_limit_ns", ctypes.c_ulonglong(int(ns)))


def wait_limit_ns() -> int:
    v = ctypes.c_ulonglong(0)
    _lib.call("se12_wait_limit_ns", ctypes.byref(v))
    return v.value


def device_status(clear: bool = True) -> int:
    """Device status word of the library (non-zero after a kernel-side error).

    After a timed-out wait (bit 0) a stream-K workspace may hold a flag that
    a late contributor set after its finisher gave up, so the pooled
    workspaces are zeroed again before any further call uses them."""
    v = ctypes.c_uint(0)
    _lib.call("se12_device_status", ctypes.byref(v), 1 if clear else 0)
    if v.value & STATUS_WAIT_TIMEOUT:
        WORKSPACES.reset()
    return v.value
