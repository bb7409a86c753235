"""ProjectionGroup's reuse rule on the CPU, with a stand-in for the segmented
matrix that counts its GEMVs: members of a group share one GEMV only for the
very input it was computed from (same storage, offset, strides, shape and
version), and the group lets go of that input once every member took it."""

from __future__ import annotations

import torch

from se12_b200.runtime import ProjectionGroup


class CountingMatrix:
    def __init__(self):
        self.calls = 0

    def gemv(self, x, out=None):
        self.calls += 1
        return x.float() * self.calls


def group():
    m = CountingMatrix()
    return m, ProjectionGroup(m, ("q", "k", "v"))


def test_members_of_one_input_share_one_gemv():
    m, g = group()
    x = torch.randn(1, 8)
    ys = [g.output(name, x) for name in ("q", "k", "v")]
    assert m.calls == 1 and ys[0] is ys[1] is ys[2]
    assert g._x is None, "the input is released once every member took the result"


def test_a_view_of_the_same_storage_counts_as_the_same_input():
    m, g = group()
    h = torch.randn(2, 8)
    g.output("q", h.reshape(-1, 8))
    g.output("k", h.reshape(-1, 8))
    assert m.calls == 1


def test_another_input_or_an_in_place_write_computes_afresh():
    m, g = group()
    x, y = torch.randn(1, 8), torch.randn(1, 8)
    g.output("q", x)
    g.output("k", y)            # another tensor: computes
    assert m.calls == 2
    g.output("q", x)
    x.mul_(2)                   # same storage, new version
    g.output("k", x)
    assert m.calls == 4
    g.output("q", x[:, :4])     # same storage, another shape
    assert m.calls == 5


def test_the_kept_input_stays_alive_while_members_are_pending():
    """The group holds the input of its kept result, so its storage cannot be
    freed and handed to another tensor before the other members ran."""
    m, g = group()
    x = torch.randn(1, 8)
    ptr = x.untyped_storage().data_ptr()
    g.output("q", x)
    del x
    assert g._x is not None and g._x.untyped_storage().data_ptr() == ptr
    g.output("k", g._x)
    g.output("v", g._x)
    assert m.calls == 1 and g._x is None


def test_a_member_called_twice_computes_again():
    m, g = group()
    x = torch.randn(1, 8)
    g.output("q", x)
    g.output("q", x)            # q already took its share: a new call
    assert m.calls == 2
