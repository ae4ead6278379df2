"""The MLP training step as Nova issues it, over any module with Fusion's API.

Mirrors the op sequence of Nova's blocks so the step runs through Fusion's
autodiff exactly as a Nova model does:
  * Linear.call: ``out = inputs @ kernel.T`` then ``out = out + bias``
    (nova/src/blocks/core/linear.py:42-48; ``.T`` is swapaxes(ndim-1, ndim-2),
    nova/src/backend/core/_tensor.py:91-98), kernel shape (units, in_features);
  * ReLU.call: ``inputs.maximum(0)`` (nova/src/blocks/activations/activations.py:9-10);
  * MeanSquaredError: ``((y_pred - y) ** 2) / size`` elementwise
    (nova/src/losses/loss_fn.py:14-15, loss.py:34-37; argument order as in
    examples/simple_network/mlp.py:65);
  * SGD (momentum 0): ``p -= grad * lr`` (nova/src/optim/sgd.py:29-44).
With data parallelism the gradients are averaged over ranks before the update; with
the backend's ``Comm`` each one is all-reduced on a second stream as soon as the
backward has completed it (``Comm.watch`` / ``Comm.collect``), overlapping the backward
of the earlier layers.
Fusion's in-place subtract reads only the parameter's count of values from the
gradient (fusion/src/Fusion/ops/Ewise.hpp:69-83), so a bias, whose gradient keeps
the batch dimension ([B, U]), moves by row 0 of it; the ranks average just those
values (``flat_prefix``), which is what the update reads, instead of shipping the
whole [B, U] gradient.
"""
from __future__ import annotations

import numpy as np


def kaiming_uniform(rng: np.random.Generator, units: int, fan_in: int) -> np.ndarray:
    bound = np.sqrt(6.0 / fan_in)
    return rng.uniform(-bound, bound, (units, fan_in)).astype(np.float32)


def init_params(dims, seed: int):
    """Kaiming-uniform kernels (units, in) and zero biases, from a numpy seed."""
    rng = np.random.default_rng(seed)
    Ws = [kaiming_uniform(rng, dims[i + 1], dims[i]) for i in range(len(dims) - 1)]
    bs = [np.zeros((dims[i + 1],), np.float32) for i in range(len(dims) - 1)]
    return Ws, bs


class MLP:
    def __init__(self, F, Ws, bs, device=None):
        self.F = F
        self.dev = device or F.CppDevice(F.CppDeviceType.CPU, 0)
        self.params = []
        for w, b in zip(Ws, bs):
            self.params.append((self.tensor(w, True), self.tensor(b, True)))

    def tensor(self, a: np.ndarray, requires_grad: bool = False):
        F = self.F
        a = np.ascontiguousarray(a, dtype=np.float32)
        return F.Tensor(list(a.shape), a.reshape(-1), F.CppDType.FLOAT32, self.dev, requires_grad)

    def forward(self, x):
        out = x
        n = len(self.params)
        for i, (W, b) in enumerate(self.params):
            out = out @ W.swapaxes(W.ndim - 1, W.ndim - 2)
            out = out + b
            if i + 1 < n:
                out = out.maximum(0)
        return out

    def step(self, x, y, lr: float, comm=None):
        """One training step; returns the loss tensor ([batch, out] elementwise MSE)."""
        F = self.F
        flat = [p for pair in self.params for p in pair]
        overlap = comm is not None and hasattr(comm, "watch")
        with F.grad_tape():
            pred = self.forward(x)
            loss = (pred - y) ** 2
            loss = loss / loss.size
            if overlap:
                comm.watch(flat)  # all-reduce each gradient as soon as the backward completes it
            loss.backward()
        if overlap:
            grads = comm.collect()
        else:
            grads = [p.get_grad() for p in flat]
            if comm is not None:
                grads = [g if g is None or g.size == p.size else self._prefix(g, p)
                         for p, g in zip(flat, grads)]
                comm.allreduce_mean([g for g in grads if g is not None])
        for p, g in zip(flat, grads):
            if g is None:
                continue
            p -= g * lr
        return loss

    def _prefix(self, g, p):
        # the values `p -= g * lr` reads from a gradient larger than p
        fp = getattr(self.F, "flat_prefix", None)
        return fp(g, p) if fp is not None else g

    def numpy_params(self):
        return [(W.to_numpy(), b.to_numpy()) for W, b in self.params]
