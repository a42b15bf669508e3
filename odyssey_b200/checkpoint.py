"""Checkpoints in the reference's on-disk layout, written from and read into a
MixedPrecisionStep.

Layout (src/odyssey/training/checkpoint.mojo:130-239, model_utils.mojo:54-97,
tensor/tensor_io.mojo:41-120):

    <dir>/checkpoint_tracker.txt              latest_epoch=<epoch>
    <dir>/checkpoint_epoch_<epoch>/<name>.weights
    <dir>/checkpoint_epoch_<epoch>/optimizer/param_<i>_slot_<j>.weights
    <dir>/checkpoint_epoch_<epoch>/optimizer/slot_counts.txt
    <dir>/checkpoint_epoch_<epoch>/metadata.txt   version=2, epoch, step, losses

A .weights file is three lines: the tensor name, "<dtype> <dim0> <dim1> ...",
and the tensor's raw bytes in memory order as lowercase hex.  Every file is
written to "<path>.tmp" and renamed (safe_write_file, utils/file_io.mojo:
572-610).  The optimizer slots per parameter are the reference's
init_*_state lists: SGD [velocity], Adam/AdamW [m, v], Lion [m],
RMSprop [square_avg, buf], Adagrad [accum].

The reference does not persist the GradientScaler; its state and the
PrecisionConfig counters go to a sidecar, mixed_precision_state.txt, which
the reference's loader never reads.

With ZeRO-1 sharding each rank writes the files of the tensors it owns; the
caller writes the shared files (metadata, slot counts, tracker) from one
rank after every rank has written (write_shared=True on that rank only).
"""
import os

import numpy as np

from . import _lib as L

_DTYPE_NAMES = {np.dtype(np.float16): "float16", np.dtype(np.float32): "float32", np.dtype(np.float64): "float64",
                np.dtype(np.int8): "int8", np.dtype(np.int16): "int16", np.dtype(np.int32): "int32",
                np.dtype(np.int64): "int64", np.dtype(np.uint8): "uint8", np.dtype(np.uint16): "uint16",
                np.dtype(np.uint32): "uint32", np.dtype(np.uint64): "uint64"}
_NAME_DTYPES = {v: k for k, v in _DTYPE_NAMES.items()}

_SLOTS = {L.SGD: ("velocity",), L.ADAM: ("m", "v"), L.ADAMW: ("m", "v"), L.LION: ("m",),
          L.RMSPROP: ("square_avg", "buf"), L.ADAGRAD: ("accum",)}


def _write_atomic(path, text):
    tmp = path + ".tmp"
    with open(tmp, "w") as f:
        f.write(text)
    os.replace(tmp, path)


def save_tensor(array, path, name="", shape=None):
    """tensor_io.mojo:41-76: name line, dtype + shape line, hex bytes line."""
    a = np.ascontiguousarray(array)
    if a.dtype not in _DTYPE_NAMES:
        raise L.OdysseyError(f"unsupported dtype {a.dtype}", L.ERR_DTYPE)
    dims = a.shape if shape is None else tuple(shape)
    if int(np.prod(dims, dtype=np.int64)) != a.size:
        raise L.OdysseyError("shape does not match the element count", L.ERR_SHAPE)
    meta = " ".join([_DTYPE_NAMES[a.dtype]] + [str(int(d)) for d in dims])
    _write_atomic(path, f"{name}\n{meta}\n{a.tobytes().hex()}\n")


def load_tensor(path):
    """tensor_io.mojo:78-120 -> (name, array shaped as stored)."""
    with open(path) as f:
        lines = f.read().split("\n")
    if len(lines) < 3:
        raise L.OdysseyError("Invalid tensor file format: expected 3+ lines", L.ERR_ARG)
    meta = lines[1].split(" ")
    if meta[0] not in _NAME_DTYPES:
        raise L.OdysseyError(f"unknown dtype {meta[0]}", L.ERR_DTYPE)
    shape = [int(x) for x in meta[1:] if x != ""]
    data = np.frombuffer(bytes.fromhex(lines[2]), _NAME_DTYPES[meta[0]])
    if data.size != int(np.prod(shape, dtype=np.int64)):
        raise L.OdysseyError("tensor file byte count does not match its shape", L.ERR_SHAPE)
    return lines[0], data.reshape(shape).copy()


def _float_text(x):
    return repr(float(np.float32(x)))


def save_checkpoint(step_ctx, checkpoint_dir, param_names, shapes, epoch, step=0, train_loss=0.0, val_loss=0.0,
                    val_acc=0.0, best_metric=float("inf"), config_snapshot="", write_shared=True):
    """CheckpointManager.save_checkpoint (checkpoint.mojo:130-239) from a
    MixedPrecisionStep: master weights as float32 parameters, the optimizer
    states as slots, metadata v2 and the tracker.  Returns the epoch
    directory."""
    n = len(step_ctx.numels)
    if len(param_names) != n or len(shapes) != n:
        raise L.OdysseyError("Parameters and param_names lists must have same length", L.ERR_ARG)
    epoch_dir = os.path.join(checkpoint_dir, f"checkpoint_epoch_{int(epoch)}")
    opt_dir = os.path.join(epoch_dir, "optimizer")
    os.makedirs(opt_dir, exist_ok=True)
    opt = int(step_ctx.cfg.optimizer)
    slots = _SLOTS[opt]
    momentum = float(step_ctx.cfg.momentum)
    for i in step_ctx.owned:
        save_tensor(step_ctx.master(i), os.path.join(epoch_dir, param_names[i] + ".weights"), param_names[i],
                    shapes[i])
        for j, slot in enumerate(slots):
            fname = f"param_{i}_slot_{j}.weights"
            has = {"velocity": momentum > 0.0, "buf": momentum > 0.0}.get(slot, True)
            val = step_ctx.state(i, 0 if j == 0 else 1) if has else np.zeros(step_ctx.numels[i], np.float32)
            save_tensor(val, os.path.join(opt_dir, fname), fname, shapes[i])
    if write_shared:
        _write_atomic(os.path.join(opt_dir, "slot_counts.txt"), "".join(f"{len(slots)}\n" for _ in range(n)))
        sc = step_ctx.scaler_state
        _write_atomic(os.path.join(epoch_dir, "mixed_precision_state.txt"),
                      "".join(f"{k}={v}\n" for k, v in sc.items()))
        meta = (f"version=2\nepoch={int(epoch)}\nstep={int(step)}\ntrain_loss={_float_text(train_loss)}\n"
                f"val_loss={_float_text(val_loss)}\nval_acc={_float_text(val_acc)}\n"
                f"best_metric={_float_text(best_metric)}\n")
        if config_snapshot:
            meta += f"config={config_snapshot}\n"
        _write_atomic(os.path.join(epoch_dir, "metadata.txt"), meta)
        _write_atomic(os.path.join(checkpoint_dir, "checkpoint_tracker.txt"), f"latest_epoch={int(epoch)}\n")
    return epoch_dir


def latest_epoch(checkpoint_dir):
    """_find_latest_epoch (checkpoint.mojo:495-523) with the partial-write
    fallback of load_latest_with_optimizer (:262-300): the newest epoch whose
    metadata.txt exists, or -1."""
    path = os.path.join(checkpoint_dir, "checkpoint_tracker.txt")
    if not os.path.exists(path):
        return -1
    latest = -1
    for line in open(path).read().split("\n"):
        if line.startswith("latest_epoch="):
            latest = int(line[len("latest_epoch="):])
            break
    for e in range(latest, -1, -1):
        if os.path.exists(os.path.join(checkpoint_dir, f"checkpoint_epoch_{e}", "metadata.txt")):
            return e
    return -1


def load_checkpoint(step_ctx, checkpoint_dir, param_names, epoch=None):
    """load_latest_with_optimizer (checkpoint.mojo:240-330) into a
    MixedPrecisionStep: this rank's master weights and optimizer slots, and
    the scaler state when the sidecar is present.  Returns (epoch, step);
    (0, 0) when there is no valid checkpoint."""
    e = latest_epoch(checkpoint_dir) if epoch is None else int(epoch)
    if e < 0:
        return 0, 0
    epoch_dir = os.path.join(checkpoint_dir, f"checkpoint_epoch_{e}")
    opt = int(step_ctx.cfg.optimizer)
    slots = _SLOTS[opt]
    momentum = float(step_ctx.cfg.momentum)
    for i in step_ctx.owned:
        _, w = load_tensor(os.path.join(epoch_dir, param_names[i] + ".weights"))
        step_ctx.set_master(i, np.ascontiguousarray(w.ravel(), np.float32))
        for j, slot in enumerate(slots):
            path = os.path.join(epoch_dir, "optimizer", f"param_{i}_slot_{j}.weights")
            if not os.path.exists(path):
                continue
            has = {"velocity": momentum > 0.0, "buf": momentum > 0.0}.get(slot, True)
            if not has:
                continue
            _, v = load_tensor(path)
            step_ctx.upload(L.BUF_STATE1 if j == 0 else L.BUF_STATE2, i, np.ascontiguousarray(v.ravel(), np.float32))
    step = 0
    meta = os.path.join(epoch_dir, "metadata.txt")
    for line in open(meta).read().split("\n"):
        if line.startswith("step="):
            step = int(line[len("step="):])
    side = os.path.join(epoch_dir, "mixed_precision_state.txt")
    if os.path.exists(side):
        kv = dict(line.split("=", 1) for line in open(side).read().split("\n") if "=" in line)
        step_ctx.set_scaler_state(float(kv["scale"]), int(kv["steps_since_growth"]), int(kv["num_steps"]),
                                  int(kv["step_count"]), int(kv["overflow_count"]))
    return e, step
