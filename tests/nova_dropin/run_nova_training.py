"""Nova's own training loop over whichever `fusion` module sits in its clib folder.

Test infrastructure. Run as a script with a copy of Nova's package on sys.path (the
copy's nova/src/backend/core/clib/ holding either the reference's pybind module or
this backend's): it builds a model from Nova's blocks exactly as Nova's example does
(InputBlock -> Linear -> ReLU -> Linear -> ReLU -> Linear, Model, MeanSquaredError,
SGD with momentum; examples/simple_network/mlp.py), overwrites the parameters with
seeded values (Nova's initialisers draw their seed from system entropy), trains a
few steps and saves the losses and parameters to the .npz named on the command line.
Nothing here re-types Nova's op sequence: the forward, loss, backward and update all
run through Nova's unchanged Python.
"""
import sys

import numpy as np


def main(out_path):
    from nova.src.backend.core import Tensor, grad_tape
    from nova.src.blocks.activations import ReLU
    from nova.src.blocks.core import InputBlock
    from nova.src.blocks.core.linear import Linear
    from nova.src.losses import MeanSquaredError
    from nova.src.models import Model
    from nova.src.optim.sgd import SGD

    inp = InputBlock((None, 16))
    x = Linear(32, "random_normal")(inp)
    x = ReLU()(x)
    x = Linear(32, "random_normal")(x)
    x = ReLU()(x)
    out = Linear(4, "random_normal")(x)
    model = Model(inputs=[inp], outputs=[out])
    params = model.parameters()
    rng = np.random.default_rng(2025)
    for p in params:
        shape = tuple(p.tensor.shape)
        scale = 1.0 / np.sqrt(shape[-1]) if len(shape) > 1 else 0.1
        p.tensor.set_values((rng.standard_normal(shape) * scale).astype(np.float32).ravel().tolist())
    optimizer = SGD(params, lr=1e-2, momentum=0.9)
    optimizer.build()
    loss_fn = MeanSquaredError()
    X = rng.standard_normal((24, 16)).astype(np.float32)
    Y = rng.standard_normal((24, 4)).astype(np.float32)
    res = {}
    for step in range(3):
        xb, yb = Tensor(X[step * 8:(step + 1) * 8 + 8]), Tensor(Y[step * 8:(step + 1) * 8 + 8])
        with grad_tape():
            y_pred = model(xb)
            loss = loss_fn(y_pred, yb)
            loss.backward()
        optimizer.step()
        res[f"step{step}.loss"] = loss.to_numpy()
        res[f"step{step}.loss_mean"] = np.asarray(loss.mean().to_numpy(), np.float32)
        for k, p in enumerate(params):
            res[f"step{step}.{p.name}{k}"] = p.tensor.to_numpy()
    np.savez(out_path, **res)


if __name__ == "__main__":
    main(sys.argv[1])
