"""Checkpoint file format (plastix_b200/checkpoint.py) on the CPU: a round
trip restores every tensor bit for bit; a file from another class, with other
fields or other shapes is refused before anything is overwritten."""
import numpy as np
import pytest
import torch

from plastix_b200.checkpoint import load_state, save_state


class Holder:
    def __init__(self, n=10, extra=False):
        g = torch.Generator().manual_seed(n)
        self.w = torch.randn(n, generator=g)
        self.ids = torch.randint(0, 1 << 30, (n,), generator=g, dtype=torch.int32)
        self.age = torch.randint(0, 256, (n,), generator=g, dtype=torch.int32).to(torch.uint8)
        self.step = 7
        self.extra = extra

    def _state_tensors(self):
        t = {"w": self.w, "ids": self.ids, "age": self.age}
        if self.extra:
            t["more"] = self.w
        return t

    def _state_meta(self):
        return {"step": self.step}

    def _load_meta(self, meta):
        self.step = meta["step"]


class Other(Holder):
    pass


def test_round_trip_bit_exact(tmp_path):
    a = Holder(100)
    save_state(a, tmp_path / "c.npz")
    b = Holder(100)
    b.w.zero_(), b.ids.zero_(), b.age.zero_()
    b.step = 0
    meta = load_state(b, tmp_path / "c.npz")
    assert meta["class"] == "Holder" and b.step == 7
    for k in ("w", "ids", "age"):
        np.testing.assert_array_equal(getattr(b, k).numpy().view(np.uint8),
                                      getattr(a, k).numpy().view(np.uint8))


def test_mismatches_are_refused(tmp_path):
    save_state(Holder(100), tmp_path / "c.npz")
    for bad, msg in ((Other(100), "written by"), (Holder(50), "field"),
                     (Holder(100, extra=True), "fields")):
        before = bad.w.clone()
        with pytest.raises(ValueError, match=msg):
            load_state(bad, tmp_path / "c.npz")
        assert torch.equal(bad.w, before)  # nothing overwritten
    np.savez(tmp_path / "x.npz", __meta__=np.array('{"format": "other"}'))
    with pytest.raises(ValueError, match="not a"):
        load_state(Holder(), tmp_path / "x.npz")
