"""Registration of the B200 kernels into einjax's own ``KernelRegistry``.

The reference dispatches sparse contractions through
``KernelRegistry.lookup(pattern, backend, sparsity)`` (``kernels/registry.py:107-140``),
whose built-ins are registered in ``KernelRegistry.__init__``
(``kernels/registry.py:63-97``). ``register_b200_kernels(registry)`` adds to
that registry (or to any object with a ``register(info)`` method and the same
``KernelInfo`` fields):

* ``b200_block_sparse_matmul`` — pattern ``"ij,jk->ik"``, backend ``"gpu"``,
  sparsity ``"sparse"``, priority 10, the signature of
  ``block_sparse_matmul_generic(lhs, rhs, block_shape=None)``;
* ``b200_sparse_einsum`` — pattern ``"*"``, same backend / sparsity /
  priority, the signature of ``execute_sparse``.

The registry's own matching rules then pick them over the generic JAX
kernels for ``backend="gpu"`` (and ``"gpu:<x>"``) lookups. Both accept the
reference's numpy relations and, with ``host_result=True``, return the
reference's ``SparseTensorRelation`` (numpy arrays, values float32), so
callers written against the reference keep working unchanged.
"""

from __future__ import annotations

from typing import Any


class _HostRelation:
    """Plain relation of numpy arrays, for callers without einjax installed."""

    def __init__(self, coords, values, shape, tile_shape):
        self.coords, self.values, self.shape, self.tile_shape = coords, values, tuple(shape), tuple(tile_shape)

    @property
    def num_tuples(self):
        return self.coords.shape[0]

    @property
    def ndim(self):
        return len(self.shape)


def _reference_attr(module: str, name: str):
    """``einjax.<module>.<name>`` when einjax is importable, else None."""
    try:
        import importlib
        return getattr(importlib.import_module(f"einjax.{module}"), name)
    except Exception:  # einjax (or jax) not installed
        return None


def _to_host(rel, relation_cls=None):
    c, v = rel.to_numpy()
    cls = relation_cls or _HostRelation
    return cls(coords=c, values=v, shape=rel.shape, tile_shape=rel.tile_shape)


def make_block_sparse_matmul_kernel(host_result=True, relation_cls=None):
    from .kernels import block_sparse_matmul_generic

    def b200_block_sparse_matmul(lhs, rhs, block_shape=None):
        res = block_sparse_matmul_generic(lhs, rhs, block_shape)
        return _to_host(res, relation_cls) if host_result else res
    return b200_block_sparse_matmul


def make_sparse_einsum_kernel(host_result=True, relation_cls=None):
    from .sparse_dispatch import execute_sparse

    def b200_sparse_einsum(lhs, rhs, join_keys, kernel_string, agg_keys, output_shape=None, output_tile_shape=None):
        res = execute_sparse(lhs, rhs, join_keys, kernel_string, agg_keys, output_shape, output_tile_shape)
        return _to_host(res, relation_cls) if host_result else res
    return b200_sparse_einsum


def register_b200_kernels(registry=None, info_cls=None, host_result=True, relation_cls=None, priority=10) -> Any:
    """Register the B200 kernels into ``registry`` and return it.

    ``registry``: einjax's ``KernelRegistry`` instance (default: a new one,
    ``einjax.kernels.registry.KernelRegistry()``) or any object with
    ``register(info)``. ``info_cls``: the registry's ``KernelInfo`` class
    (default: einjax's). ``relation_cls``: class of host results (default:
    einjax's ``SparseTensorRelation``, else a plain numpy-holding relation).
    """
    if registry is None:
        cls = _reference_attr("kernels.registry", "KernelRegistry")
        if cls is None:
            raise ImportError("einjax is not importable: pass the registry to register into")
        registry = cls()
    info_cls = info_cls or _reference_attr("kernels.registry", "KernelInfo")
    if info_cls is None:
        raise ImportError("einjax is not importable: pass the registry's KernelInfo class as info_cls")
    if relation_cls is None and host_result:
        relation_cls = _reference_attr("tensor.sparse", "SparseTensorRelation")
    registry.register(info_cls(name="b200_block_sparse_matmul", pattern="ij,jk->ik", backend="gpu",
                               sparsity="sparse", priority=priority,
                               kernel_fn=make_block_sparse_matmul_kernel(host_result, relation_cls)))
    registry.register(info_cls(name="b200_sparse_einsum", pattern="*", backend="gpu", sparsity="sparse",
                               priority=priority, kernel_fn=make_sparse_einsum_kernel(host_result, relation_cls)))
    return registry
