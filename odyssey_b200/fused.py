"""MixedPrecisionStep: the fused, device-resident update path.

Replaces the per-tensor call sequence of the reference's drivers
(examples/lenet_emnist/run_train.mojo:219-306,
examples/mixed_precision_training.mojo:132-216): unscale -> finite check ->
[skip + backoff] -> global-norm clip -> SGD/Adam/AdamW on float32 master
weights -> requant -> scaler step, as one ody_step call of libodyssey_mp.so.
Parameters, states and gradients live in device arenas owned by the
context; with world_size > 1 whole tensors are sharded across ranks
(ZeRO-1) and only a 16-byte {nonfinite, sumsq} pair per rank crosses NVLink.
"""
import ctypes as C

import numpy as np

from . import _lib as L
from .quant import QuantizedTensor

_OPT = {"sgd": L.SGD, "adam": L.ADAM, "adamw": L.ADAMW, "lion": L.LION, "rmsprop": L.RMSPROP,
        "adagrad": L.ADAGRAD}
_GDT = {"float32": L.F32, "float16": L.F16, "bfloat16": L.BF16}
# where the apply kernel runs the per-tensor-scaled kinds' requant jobs
# (ody_config.requant_placement); results are identical under each
_PLACEMENT = {"auto": 0, "interleaved": 1, "at_end": 2}


def nccl_unique_id():
    buf = (C.c_char * 128)()
    L.check(L.lib().ody_nccl_unique_id(buf))
    return bytes(buf)


def plan_shards(numels, world_size):
    """Host-only ZeRO-1 plan: owner rank of each tensor (ody_plan_shards)."""
    n = np.ascontiguousarray(numels, np.int64)
    out = np.zeros(max(len(n), 1), np.int32)
    L.check(L.lib().ody_plan_shards(n.ctypes.data, len(n), world_size, out.ctypes.data))
    return out[: len(n)].tolist()


class MixedPrecisionStep:
    def __init__(self, numels, grad_dtype="bfloat16", quant="none", optimizer="adamw", learning_rate=1e-3,
                 momentum=0.0, beta1=0.9, beta2=0.999, epsilon=1e-8, weight_decay=0.0,
                 use_gradient_scaler=True, initial_scale=65536.0, growth_factor=2.0, backoff_factor=0.5,
                 growth_interval=2000, min_scale=1.0, max_scale=65536.0, clip_max_norm=None, device=0,
                 world_size=1, rank=0, unique_id=None, comm_timeout_ms=60000, alpha=0.99, chunk_elems=0,
                 requant_placement="auto"):
        cfg = L.default_config()
        cfg.optimizer = _OPT[optimizer] if isinstance(optimizer, str) else int(optimizer)
        cfg.device = int(device)
        cfg.learning_rate, cfg.momentum = learning_rate, momentum
        cfg.beta1, cfg.beta2, cfg.epsilon, cfg.weight_decay = beta1, beta2, epsilon, weight_decay
        cfg.use_gradient_scaler = int(bool(use_gradient_scaler))
        cfg.initial_scale, cfg.growth_factor, cfg.backoff_factor = initial_scale, growth_factor, backoff_factor
        cfg.growth_interval, cfg.min_scale, cfg.max_scale = growth_interval, min_scale, max_scale
        cfg.clip_enabled = int(clip_max_norm is not None)
        cfg.max_norm = float(clip_max_norm) if clip_max_norm is not None else 1.0
        cfg.comm_timeout_ms = int(comm_timeout_ms)
        cfg.alpha = float(alpha)
        cfg.chunk_elems = int(chunk_elems)
        cfg.requant_placement = (_PLACEMENT[requant_placement] if isinstance(requant_placement, str)
                                 else int(requant_placement))
        self.cfg = cfg
        self.numels = [int(n) for n in numels]
        self.grad_dtype = _GDT[grad_dtype] if isinstance(grad_dtype, str) else int(grad_dtype)
        quants = quant if isinstance(quant, (list, tuple)) else [quant] * len(self.numels)
        self.quants = [L.QUANT_NAMES[q] if isinstance(q, str) else int(q) for q in quants]
        self.world_size, self.rank = int(world_size), int(rank)
        self._ctx = C.c_void_p()
        L.check(L.lib().ody_ctx_create(C.byref(self._ctx), C.byref(cfg)))
        try:
            for n, q in zip(self.numels, self.quants):
                L.check(L.lib().ody_ctx_add_tensor(self._ctx, n, self.grad_dtype, q, None), self._ctx)
            uid = None
            if self.world_size > 1:
                if unique_id is None or len(unique_id) != 128:
                    raise L.OdysseyError("a 128-byte NCCL unique id is required for world_size > 1")
                uid = C.create_string_buffer(bytes(unique_id), 128)
            L.check(L.lib().ody_ctx_finalize(self._ctx, self.world_size, self.rank, uid), self._ctx)
        except Exception:
            self.close()
            raise
        self.owner = plan_shards(self.numels, self.world_size)
        self.owned = [i for i, r in enumerate(self.owner) if r == self.rank]

    @classmethod
    def from_process_group(cls, numels, group=None, **kw):
        """Build on every rank of a torch.distributed group (the group only
        carries the NCCL unique id; the step itself uses NCCL directly)."""
        import torch.distributed as dist
        rank, world = dist.get_rank(group), dist.get_world_size(group)
        obj = [nccl_unique_id() if rank == 0 and world > 1 else None]
        if world > 1:
            dist.broadcast_object_list(obj, src=0, group=group)
        return cls(numels, world_size=world, rank=rank, unique_id=obj[0], **kw)

    # ---- buffers ----
    def _esz(self, which):
        if which not in (L.BUF_GRAD, L.BUF_DP_GRAD):
            return 4
        return 4 if self.grad_dtype == L.F32 else 2

    def upload(self, which, index, array, sync=True):
        a = L.contiguous(array)
        fn = L.lib().ody_upload if sync else L.lib().ody_upload_async
        L.check(fn(self._ctx, which, index, L.ptr(a), L.numel(a) * self._esz(which)), self._ctx)
        return a

    def download(self, which, index, out=None):
        n = self.numels[index]
        if out is None:
            out = np.empty(n, np.float32 if self._esz(which) == 4 else np.uint16)
        L.check(L.lib().ody_download(self._ctx, which, index, L.ptr(out), n * self._esz(which)), self._ctx)
        return out

    def set_master(self, i, a):
        return self.upload(L.BUF_MASTER, i, a)

    def set_grad(self, i, a, sync=True):
        return self.upload(L.BUF_GRAD, i, a, sync)

    def master(self, i):
        return self.download(L.BUF_MASTER, i)

    def state(self, i, k):
        return self.download(L.BUF_STATE1 if k == 0 else L.BUF_STATE2, i)

    def device_ptr(self, which, i):
        p = C.c_void_p()
        L.check(L.lib().ody_ctx_device_ptr(self._ctx, which, i, C.byref(p)), self._ctx)
        return p.value

    def get_quant(self, i, out=None):
        nb = L.quant_bytes(self.quants[i], self.numels[i])
        if out is None:
            out = np.empty(nb, np.uint8)
        ts = C.c_float(1.0)
        L.check(L.lib().ody_get_quant(self._ctx, i, L.ptr(out), nb, C.byref(ts)), self._ctx)
        return QuantizedTensor(out, self.quants[i], self.numels[i], ts.value)

    def quant_layout(self, i=-1):
        """(offset, bytes, total) of tensor i in the gathered quantised model."""
        off, nb, tot = C.c_int64(0), C.c_int64(0), C.c_int64(0)
        L.check(L.lib().ody_ctx_quant_layout(self._ctx, i, C.byref(off), C.byref(nb), C.byref(tot)), self._ctx)
        return off.value, nb.value, tot.value

    def gather_quant(self):
        """The whole model's quantised weights on this rank's GPU (collective):
        (uint8 CUDA tensor in quant_layout order, float32 CUDA tensor of the
        per-tensor scales)."""
        import torch
        total = self.quant_layout()[2]
        dev = torch.device("cuda", self.cfg.device)
        buf = torch.empty(max(total, 1), dtype=torch.uint8, device=dev)
        scales = torch.empty(max(len(self.numels), 1), dtype=torch.float32, device=dev)
        L.check(L.lib().ody_ctx_gather_quant(self._ctx, buf.data_ptr(), scales.data_ptr()), self._ctx)
        return buf, scales

    # ---- the step ----
    def step(self, t=1):
        r = L.StepResult()
        L.check(L.lib().ody_step(self._ctx, int(t), C.byref(r)), self._ctx)
        return r.as_dict()

    def step_async(self, t=1):
        L.check(L.lib().ody_step_async(self._ctx, int(t)), self._ctx)

    def wait(self):
        r = L.StepResult()
        L.check(L.lib().ody_step_wait(self._ctx, C.byref(r)), self._ctx)
        return r.as_dict()

    def set_timing(self, enable=True):
        L.check(L.lib().ody_ctx_set_timing(self._ctx, int(bool(enable))), self._ctx)

    def dp_attach(self):
        """Data-parallel gradients (collective; see ody_ctx_dp_attach): every
        rank fills its full-model gradients with set_dp_grad, and each step
        reduce-scatters them (rank-order float32 sum) fused with pass 1."""
        L.check(L.lib().ody_ctx_dp_attach(self._ctx), self._ctx)

    def set_dp_grad(self, i, a, sync=True):
        """This rank's gradient of tensor i (any tensor) in the data-parallel
        buffer."""
        return self.upload(L.BUF_DP_GRAD, i, a, sync)

    def set_graph(self, enable=True):
        """Replay each step as one CUDA graph launch (one GPU; see
        ody_ctx_set_graph)."""
        L.check(L.lib().ody_ctx_set_graph(self._ctx, int(bool(enable))), self._ctx)

    def set_grad_double_buffer(self, enable=True):
        """Two gradient arenas, alternating per step: set_grad(..., sync=False)
        for step t+1 right after step_async(t) copies on a separate stream
        while step t runs (see ody_ctx_set_grad_double_buffer)."""
        L.check(L.lib().ody_ctx_set_grad_double_buffer(self._ctx, int(bool(enable))), self._ctx)

    def pass_times(self):
        """{'stats','exchange','update','requant'} milliseconds accumulated over
        the timed steps since the last call, and the step count."""
        ms = (C.c_double * 4)()
        n = C.c_int64(0)
        L.check(L.lib().ody_ctx_pass_times(self._ctx, ms, C.byref(n)), self._ctx)
        return dict(zip(("stats", "exchange", "update", "requant"), list(ms))), n.value

    def stream_handle(self):
        s = C.c_void_p()
        L.check(L.lib().ody_ctx_stream(self._ctx, C.byref(s)), self._ctx)
        return s.value

    @property
    def scaler_state(self):
        s, a, b, c, d = C.c_float(), C.c_int64(), C.c_int64(), C.c_int64(), C.c_int64()
        L.check(L.lib().ody_get_scaler(self._ctx, C.byref(s), C.byref(a), C.byref(b), C.byref(c), C.byref(d)),
                self._ctx)
        return {"scale": s.value, "steps_since_growth": a.value, "num_steps": b.value, "step_count": c.value,
                "overflow_count": d.value}

    def set_scaler_state(self, scale, steps_since_growth=0, num_steps=0, step_count=0, overflow_count=0):
        L.check(L.lib().ody_set_scaler(self._ctx, scale, steps_since_growth, num_steps, step_count,
                                       overflow_count), self._ctx)

    def export_state(self):
        n = C.c_size_t(0)
        L.check(L.lib().ody_ctx_export(self._ctx, None, C.byref(n)), self._ctx)
        buf = np.empty(n.value, np.uint8)
        L.check(L.lib().ody_ctx_export(self._ctx, buf.ctypes.data, C.byref(n)), self._ctx)
        return buf.tobytes()

    def import_state(self, blob):
        b = np.frombuffer(blob, np.uint8)
        L.check(L.lib().ody_ctx_import(self._ctx, b.ctypes.data, b.size), self._ctx)

    def close(self):
        if getattr(self, "_ctx", None) and self._ctx.value:
            L.lib().ody_ctx_destroy(self._ctx)
            self._ctx = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
