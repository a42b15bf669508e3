"""The reference's checkpoint layout (training/checkpoint.mojo:130-330,
tensor/tensor_io.mojo:41-120) written and read by odyssey_b200.checkpoint:
exact file text, slot layout per optimizer, partial-write recovery, and a
round trip through a host-side stand-in for the step context (no GPU)."""
import os

import numpy as np
import pytest

from odyssey_b200 import _lib as L
from odyssey_b200 import checkpoint as ck


def test_weights_file_text(tmp_path):
    p = tmp_path / "w.weights"
    ck.save_tensor(np.array([1.0, -2.0], np.float32), str(p), "conv1_kernel", (1, 2))
    # name, "dtype dims", raw bytes in memory order (little endian) as hex
    assert p.read_text() == "conv1_kernel\nfloat32 1 2\n0000803f000000c0\n"
    name, a = ck.load_tensor(str(p))
    assert name == "conv1_kernel" and a.shape == (1, 2) and a.dtype == np.float32
    np.testing.assert_array_equal(a, [[1.0, -2.0]])
    assert not os.path.exists(str(p) + ".tmp")


def test_bad_files(tmp_path):
    p = tmp_path / "x.weights"
    p.write_text("only\n")
    with pytest.raises(L.OdysseyError, match="expected 3\\+ lines"):
        ck.load_tensor(str(p))
    p.write_text("n\nfloat32 3\n0000803f\n")
    with pytest.raises(L.OdysseyError, match="byte count"):
        ck.load_tensor(str(p))


class FakeCtx:
    """The part of MixedPrecisionStep the checkpoint module uses, on host arrays."""

    def __init__(self, numels, optimizer, momentum=0.0, owned=None):
        class Cfg:
            pass
        self.cfg = Cfg()
        self.cfg.optimizer, self.cfg.momentum = optimizer, momentum
        self.numels = numels
        self.owned = list(range(len(numels))) if owned is None else owned
        self.m = {i: np.zeros(n, np.float32) for i, n in enumerate(numels)}
        self.s = {(i, k): np.zeros(n, np.float32) for i, n in enumerate(numels) for k in (0, 1)}
        self.scaler_state = {"scale": 65536.0, "steps_since_growth": 0, "num_steps": 0, "step_count": 0,
                             "overflow_count": 0}

    def master(self, i):
        return self.m[i].copy()

    def state(self, i, k):
        return self.s[(i, k)].copy()

    def set_master(self, i, a):
        self.m[i][:] = a

    def upload(self, which, i, a):
        self.s[(i, 0 if which == L.BUF_STATE1 else 1)][:] = a

    def set_scaler_state(self, scale, a, b, c, d):
        self.scaler_state = {"scale": scale, "steps_since_growth": a, "num_steps": b, "step_count": c,
                             "overflow_count": d}


@pytest.mark.parametrize("opt,momentum,slots", [(L.SGD, 0.9, 1), (L.SGD, 0.0, 1), (L.ADAMW, 0.0, 2), (L.LION, 0.0, 1),
                                                (L.RMSPROP, 0.9, 2), (L.RMSPROP, 0.0, 2), (L.ADAGRAD, 0.0, 1)])
def test_round_trip(tmp_path, opt, momentum, slots):
    rng = np.random.default_rng(3)
    names, shapes = ["conv_w", "conv_b", "fc_w"], [(2, 3, 2), (2,), (4, 5)]
    a = FakeCtx([12, 2, 20], opt, momentum)
    for i, n in enumerate(a.numels):
        a.m[i][:] = rng.standard_normal(n)
        a.s[(i, 0)][:] = rng.standard_normal(n)
        a.s[(i, 1)][:] = rng.standard_normal(n)
    a.scaler_state = {"scale": 1024.0, "steps_since_growth": 7, "num_steps": 11, "step_count": 12,
                      "overflow_count": 1}
    d = ck.save_checkpoint(a, str(tmp_path), names, shapes, epoch=3, step=140, train_loss=0.5, val_loss=0.25,
                           val_acc=0.75, best_metric=0.25, config_snapshot="epochs=50|batch_size=64")
    assert (tmp_path / "checkpoint_tracker.txt").read_text() == "latest_epoch=3\n"
    assert (tmp_path / "checkpoint_epoch_3" / "optimizer" / "slot_counts.txt").read_text() == f"{slots}\n" * 3
    meta = (tmp_path / "checkpoint_epoch_3" / "metadata.txt").read_text().split("\n")
    assert meta[:3] == ["version=2", "epoch=3", "step=140"] and "config=epochs=50|batch_size=64" in meta
    _, w = ck.load_tensor(os.path.join(d, "fc_w.weights"))
    assert w.shape == (4, 5)
    b = FakeCtx([12, 2, 20], opt, momentum)
    assert ck.load_checkpoint(b, str(tmp_path), names) == (3, 140)
    for i in range(3):
        np.testing.assert_array_equal(b.m[i], a.m[i])
        uses_s1 = not (opt == L.SGD and momentum == 0.0)
        uses_s2 = opt in (L.ADAM, L.ADAMW) or (opt == L.RMSPROP and momentum > 0.0)
        np.testing.assert_array_equal(b.s[(i, 0)], a.s[(i, 0)] if uses_s1 else 0.0)
        np.testing.assert_array_equal(b.s[(i, 1)], a.s[(i, 1)] if uses_s2 else 0.0)
    assert b.scaler_state == a.scaler_state


def test_partial_write_falls_back(tmp_path):
    """load_latest_with_optimizer's recovery: a tracker epoch without
    metadata.txt falls back to the newest complete one."""
    a = FakeCtx([4], L.ADAMW)
    a.m[0][:] = 1.0
    ck.save_checkpoint(a, str(tmp_path), ["w"], [(4,)], epoch=1, step=10)
    a.m[0][:] = 2.0
    ck.save_checkpoint(a, str(tmp_path), ["w"], [(4,)], epoch=2, step=20)
    os.remove(tmp_path / "checkpoint_epoch_2" / "metadata.txt")
    assert ck.latest_epoch(str(tmp_path)) == 1
    b = FakeCtx([4], L.ADAMW)
    assert ck.load_checkpoint(b, str(tmp_path), ["w"]) == (1, 10)
    np.testing.assert_array_equal(b.m[0], 1.0)
    assert ck.load_checkpoint(FakeCtx([4], L.ADAMW), str(tmp_path / "none"), ["w"]) == (0, 0)


def test_sharded_ranks_write_disjoint_files(tmp_path):
    """Each rank writes its own tensors; the shared files come from one rank."""
    r0 = FakeCtx([4, 4], L.ADAMW, owned=[0])
    r1 = FakeCtx([4, 4], L.ADAMW, owned=[1])
    r0.m[0][:] = 1.0
    r1.m[1][:] = 2.0
    ck.save_checkpoint(r1, str(tmp_path), ["a", "b"], [(4,), (4,)], epoch=0, write_shared=False)
    ck.save_checkpoint(r0, str(tmp_path), ["a", "b"], [(4,), (4,)], epoch=0, write_shared=True)
    whole = FakeCtx([4, 4], L.ADAMW)
    ck.load_checkpoint(whole, str(tmp_path), ["a", "b"])
    np.testing.assert_array_equal(whole.m[0], 1.0)
    np.testing.assert_array_equal(whole.m[1], 2.0)
