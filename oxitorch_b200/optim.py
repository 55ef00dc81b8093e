"""Optimizers with their math and state on the GPU: the reference's
``oxitorch.optim`` ``Sgd`` / ``AdamW`` / ``Adam`` (python/oxitorch/optim.py:18-99,
over ``_native.RustSgd`` / ``RustAdamW``, crates/oxi-bindings/src/lib.rs:833-930)
with the same constructor arguments, defaults, ``lr`` property, ``zero_grad()`` /
``step()`` and errors.

Each ``step()`` launches one kernel per parameter that has a gradient
(``oxc_sgd_step`` / ``oxc_adamw_step``), which updates the parameter in place
with the reference's per-element f32 arithmetic (crates/oxi-autograd/src/optim.rs),
so values match the reference bit for bit.  State -- velocity buffers, Adam
moments, per-parameter step counters -- lives on the device, created lazily per
parameter index on that parameter's first gradient, like the reference's slots:
a parameter without a gradient is skipped and keeps its state and counter.

Parameters are float32 CUDA tensors (``.grad`` as autograd leaves them);
hyperparameters are rounded to f32 as the reference's constructors do.
"""

from __future__ import annotations

import numpy as np
import torch

from . import _native as N


def _f32(x) -> float:
    return float(np.float32(x))


class _DeviceOptimizer:
    """Shared plumbing: the parameter list, the f32 learning rate, per-index
    lazily created state (``_slot``) and ``zero_grad`` / ``step``."""

    def __init__(self, params, lr):
        self.params = list(params)
        self._lr = _f32(lr)
        self._slots: list[dict | None] = []

    @staticmethod
    def _tensors(params):
        """Accepts wrappers with a ``.tensor`` attribute and bare tensors."""
        return [p.tensor if hasattr(p, "tensor") else p for p in params]

    @property
    def lr(self):
        return self._lr

    @lr.setter
    def lr(self, value):
        self._lr = _f32(value)  # stored as f32 (lib.rs:854-860, 907-913)

    def zero_grad(self):
        """Sets every gradient to zeros (graph.rs:229-233 stores a zero
        tensor, so the next step still counts for Adam's bias correction)."""
        for p in self._tensors(self.params):
            if p.grad is None:
                p.grad = torch.zeros_like(p)
            else:
                p.grad.zero_()

    def step(self):
        for index, p in enumerate(self._tensors(self.params)):
            if p.grad is None:
                continue
            self._check(index, p)
            self._step_param(index, p, p.grad.contiguous())

    @staticmethod
    def _check(index, p):
        if not isinstance(p, torch.Tensor) or not p.is_cuda or p.dtype != torch.float32:
            raise ValueError(f"invalid argument: parameter {index} must be a float32 CUDA "
                             "tensor (oxitorch_b200 has no CPU path)")
        if not p.is_contiguous():
            raise ValueError(f"invalid argument: parameter {index} must be contiguous")
        if p.grad.shape != p.shape:
            raise ValueError(f"invalid argument: parameter {index} and its gradient differ in "
                             f"shape: {tuple(p.shape)} vs {tuple(p.grad.shape)}")

    def _slot(self, index, p, names):
        """The state dict of parameter ``index``: zero buffers ``names`` and a
        step counter, created on first use; the reference's error if the
        parameter's size changed (optim.rs:33-51)."""
        while len(self._slots) <= index:
            self._slots.append(None)
        st = self._slots[index]
        if st is None:
            st = {k: torch.zeros(p.numel(), dtype=torch.float32, device=p.device) for k in names}
            st["step"] = 0
            self._slots[index] = st
        n = p.numel()
        for k in names:
            if st[k].numel() != n:
                raise ValueError(
                    f"invalid argument: optimizer state for parameter {index} has "
                    f"{st[k].numel()} elements but the parameter now has {n}; the parameter "
                    "set changed mid-run")
        return st


class Sgd(_DeviceOptimizer):
    """Vanilla SGD with optional (Nesterov) momentum (optim.rs:62-138); the
    velocity starts at zero on a parameter's first gradient, so its first
    buffer is that gradient."""

    def __init__(self, params, lr=0.01, momentum=0.0, nesterov=False):
        if nesterov and momentum <= 0.0:
            raise ValueError("nesterov momentum requires momentum > 0")
        self.momentum = momentum
        self.nesterov = nesterov
        super().__init__(params, lr)

    def _step_param(self, index, p, g):
        L = N.load()
        mom = _f32(self.momentum)
        vel = None
        if mom > 0.0:
            vel = self._slot(index, p, ("velocity",))["velocity"]
        N.check(L.oxc_sgd_step(p.data_ptr(), g.data_ptr(), None if vel is None else vel.data_ptr(),
                               p.numel(), self._lr, mom, int(bool(self.nesterov)),
                               torch.cuda.current_stream(p.device).cuda_stream), "sgd step")


class _Adam(_DeviceOptimizer):
    def __init__(self, params, lr, betas, eps, weight_decay, decoupled):
        self.betas = tuple(betas)
        self.eps = eps
        self.weight_decay = weight_decay
        self._decoupled = decoupled
        super().__init__(params, lr)

    def _step_param(self, index, p, g):
        L = N.load()
        st = self._slot(index, p, ("m", "v"))
        st["step"] += 1  # bump_step (optim.rs:54-60): only when there is a gradient
        N.check(L.oxc_adamw_step(p.data_ptr(), g.data_ptr(), st["m"].data_ptr(),
                                 st["v"].data_ptr(), p.numel(), self._lr, _f32(self.betas[0]),
                                 _f32(self.betas[1]), _f32(self.eps), _f32(self.weight_decay),
                                 int(self._decoupled), st["step"],
                                 torch.cuda.current_stream(p.device).cuda_stream), "adam step")


class AdamW(_Adam):
    """AdamW (Loshchilov & Hutter, 2019): decay applied to the parameter.
    Defaults as the reference: lr 1e-3, betas (0.9, 0.999), eps 1e-8,
    weight_decay 1e-2."""

    def __init__(self, params, lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=1e-2):
        super().__init__(params, lr, betas, eps, weight_decay, True)


class Adam(_Adam):
    """Adam (Kingma & Ba, 2015): decay added to the gradient before the
    moments.  Defaults as the reference: weight_decay 0."""

    def __init__(self, params, lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.0):
        super().__init__(params, lr, betas, eps, weight_decay, False)
