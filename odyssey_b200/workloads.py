"""Synthetic workloads of the five benchmark configurations (shapes, seeded
value distributions, hyper-parameters).  No dataset or checkpoint is
involved: every input is drawn from numpy's PCG64 with a fixed seed.

1 LeNet-5 (61,706 params, FP16 grads x 1024, SGD mu=0.9 lr=0.01 wd=5e-4, FP16 out)
2 MXFP4 quant+dequant of a 4096x4096 float32 N(0,1) tensor, 0.1 % outliers x100
3 NVFP4 requant of an 8192x8192 bfloat16 N(0,0.02^2) tensor, 0.05 % outliers x50
4 ResNet-18 CIFAR (62 tensors, 11,173,962 params) AdamW, BF16 grads x 65536,
  inf injected every 100th step, FP8-E4M3 per-tensor scale
5 1B flat: 64 x 4096x4096, AdamW + global-norm clip 1.0, BF16 grads x 4096,
  NVFP4 with per-tensor scale
"""
import numpy as np

LENET_SHAPES = [(6, 1, 5, 5), (6,), (16, 6, 5, 5), (16,), (120, 400), (120,), (84, 120), (84,), (10, 84), (10,)]


def resnet18_cifar_shapes(num_classes=10):
    """torchvision-style BasicBlock [2,2,2,2], 3x3 stem, no conv bias, BN gamma/beta."""
    shapes = [(64, 3, 3, 3), (64,), (64,)]
    cin = 64
    for cout, stride in ((64, 1), (128, 2), (256, 2), (512, 2)):
        for b in range(2):
            s = stride if b == 0 else 1
            shapes += [(cout, cin, 3, 3), (cout,), (cout,), (cout, cout, 3, 3), (cout,), (cout,)]
            if b == 0 and (s != 1 or cin != cout):
                shapes += [(cout, cin, 1, 1), (cout,), (cout,)]
            cin = cout
    shapes += [(num_classes, 512), (num_classes,)]
    return shapes


RESNET18_SHAPES = resnet18_cifar_shapes()
FLAT1B_SHAPES = [(4096, 4096)] * 64


def numels(shapes):
    return [int(np.prod(s)) for s in shapes]


def f32_to_bf16_bits(x):
    """Round-to-nearest-even float32 -> bfloat16 bit patterns (finite inputs)."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32)
    r = (u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))) >> np.uint32(16)
    return r.astype(np.uint16)


def bf16_bits_to_f32(h):
    return (np.asarray(h, np.uint16).astype(np.uint32) << np.uint32(16)).view(np.float32)


class Workload:
    """Model description + seeded generators for one configuration."""

    def __init__(self, name, shapes, grad_dtype, quant, optimizer, hyper, master_std, grad_std, loss_scale,
                 clip=None, inf_every=0, scaler=None):
        self.name, self.shapes = name, shapes
        self.numels = numels(shapes)
        self.grad_dtype, self.quant, self.optimizer = grad_dtype, quant, optimizer
        self.hyper = hyper
        self.master_std, self.grad_std, self.loss_scale = master_std, grad_std, loss_scale
        self.clip, self.inf_every = clip, inf_every
        self.scaler = scaler or {}

    @property
    def total(self):
        return sum(self.numels)

    def master(self, seed=0, scale_numels=None):
        rng = np.random.Generator(np.random.PCG64(seed))
        return [(rng.standard_normal(n, dtype=np.float32) * np.float32(self.master_std)) for n in
                (scale_numels or self.numels)]

    def grads(self, step, seed=1, scale_numels=None):
        """Scaled low-precision gradients of one step (uint16 bf16 bits,
        float16, or float32)."""
        rng = np.random.Generator(np.random.PCG64([seed, step]))
        out = []
        nl = scale_numels or self.numels
        for n in nl:
            g = rng.standard_normal(n, dtype=np.float32) * np.float32(self.grad_std) * np.float32(self.loss_scale)
            if self.grad_dtype == "bfloat16":
                out.append(f32_to_bf16_bits(g))
            elif self.grad_dtype == "float16":
                out.append(g.astype(np.float16))
            else:
                out.append(g)
        if self.inf_every and step > 0 and step % self.inf_every == 0:
            t = int(rng.integers(len(nl)))
            i = int(rng.integers(nl[t]))
            inf = {"bfloat16": np.uint16(0x7F80), "float16": np.float16(np.inf), "float32": np.float32(np.inf)}
            out[t][i] = inf[self.grad_dtype]
        return out

    def step_kwargs(self):
        kw = dict(grad_dtype=self.grad_dtype, quant=self.quant, optimizer=self.optimizer, **self.hyper)
        kw.update(self.scaler)
        kw["initial_scale"] = float(self.loss_scale)
        if self.clip is not None:
            kw["clip_max_norm"] = self.clip
        return kw


def lenet():
    return Workload("lenet5_sgd_fp16", LENET_SHAPES, "float16", "fp16", "sgd",
                    dict(learning_rate=0.01, momentum=0.9, weight_decay=5e-4), 0.05, 1e-3, 1024.0)


def resnet18():
    return Workload("resnet18_adamw_bf16_fp8", RESNET18_SHAPES, "bfloat16", "fp8_tensor", "adamw",
                    dict(learning_rate=1e-3, beta1=0.9, beta2=0.999, epsilon=1e-8, weight_decay=0.01),
                    0.02, 1e-4, 65536.0, inf_every=100,
                    scaler=dict(growth_factor=2.0, backoff_factor=0.5, growth_interval=2000, min_scale=1.0,
                                max_scale=65536.0))


def flat1b(ntensors=64, side=4096):
    return Workload("flat1b_adamw_clip_bf16_nvfp4", [(side, side)] * ntensors, "bfloat16", "nvfp4_tensor",
                    "adamw", dict(learning_rate=1e-3, beta1=0.9, beta2=0.999, epsilon=1e-8, weight_decay=0.01),
                    0.02, 1e-3, 4096.0, clip=1.0)


def mxfp4_tensor(seed=0, side=4096):
    """Config 2 input: N(0,1), 0.1 % of positions (without replacement) x100."""
    rng = np.random.Generator(np.random.PCG64(seed))
    n = side * side
    x = rng.standard_normal(n, dtype=np.float32)
    pos = rng.choice(n, size=n // 1000, replace=False)
    x[pos] *= np.float32(100.0)
    return x


def nvfp4_tensor_bf16(seed=0, side=8192):
    """Config 3 input: bf16 RNE(N(0,0.02^2)), 0.05 % of positions x50."""
    rng = np.random.Generator(np.random.PCG64(seed))
    n = side * side
    x = rng.standard_normal(n, dtype=np.float32) * np.float32(0.02)
    pos = rng.choice(n, size=n // 2000, replace=False)
    x[pos] *= np.float32(50.0)
    return f32_to_bf16_bits(x)
