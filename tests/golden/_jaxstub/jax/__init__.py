"""Numpy stand-in for the parts of ``jax`` that einjax's sparse path touches.

Used only by ``tests/golden/make_golden.py`` to run the unmodified reference
modules in a container without jaxlib. ``jax.numpy`` maps onto numpy; ``jit``
is the identity; ``custom_vjp`` records its fwd/bwd so the generator can call
the reference's own backward rule; sharding objects are inert placeholders
and ``device_put``/``device_get`` are the identity.

``F32`` switches ``jnp.array`` to JAX's default x64-off behaviour (float64
input becomes float32).
"""

import numpy as _np

from . import numpy  # noqa: F401
from . import sharding  # noqa: F401

F32 = False
Array = _np.ndarray
LAST_VJP = []


class _Stages:
    Compiled = object


stages = _Stages()


def jit(fun=None, **kwargs):
    if fun is None:
        return lambda f: f
    return fun


class custom_vjp:
    def __init__(self, fun):
        self.fun = fun
        self.fwd = None
        self.bwd = None
        LAST_VJP.append(self)

    def defvjp(self, fwd, bwd):
        self.fwd, self.bwd = fwd, bwd

    def __call__(self, *args):
        return self.fun(*args)


class _Device:
    def __init__(self, i):
        self.id = i
        self.platform = "cpu"


NUM_FAKE_DEVICES = 1


def devices():
    return [_Device(i) for i in range(NUM_FAKE_DEVICES)]


def local_devices():
    return devices()


def device_put(x, sharding=None):
    return x


def device_get(x):
    return x
