"""numpy-backed ``jax.numpy`` for the golden-vector generator."""

import numpy as _np

import jax as _jax

ndarray = _np.ndarray
float32 = _np.float32
float64 = _np.float64
int32 = _np.int32


class _AtArray(_np.ndarray):
    """ndarray with a functional ``.at[idx].add(v)`` like jax arrays."""

    @property
    def at(self):
        arr = self

        class _Idx:
            def __getitem__(self, idx):
                class _Op:
                    def add(self, v):
                        out = _np.array(arr).view(_AtArray)
                        _np.add.at(out, idx, v)
                        return out
                return _Op()
        return _Idx()


def array(x, dtype=None):
    a = _np.array(x, dtype=dtype)
    if dtype is None and _jax.F32 and a.dtype == _np.float64:
        a = a.astype(_np.float32)
    return a.view(_AtArray)


def asarray(x, dtype=None):
    return array(x, dtype)


def einsum(s, *ops):
    return _np.asarray(_np.einsum(s, *[_np.asarray(o) for o in ops])).view(_AtArray)


def zeros(shape, dtype=None):
    return _np.zeros(shape, dtype=dtype if dtype is not None else
                     (_np.float32 if _jax.F32 else _np.float64)).view(_AtArray)


def zeros_like(x):
    return _np.zeros_like(_np.asarray(x)).view(_AtArray)


def concatenate(xs, axis=0):
    return _np.concatenate([_np.asarray(x) for x in xs], axis=axis).view(_AtArray)


def sum(x, *a, **k):  # noqa: A001
    return _np.sum(_np.asarray(x), *a, **k)


all = _np.all  # noqa: A001
isfinite = _np.isfinite
