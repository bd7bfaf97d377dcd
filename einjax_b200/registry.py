"""Kernel registry; mirrors einjax ``kernels/registry.py`` and registers the
B200 kernels into it.

``KernelRegistry``/``KernelInfo`` keep the reference's lookup rules
(``kernels/registry.py:27-273``): highest priority wins, ``"*"`` matches any
pattern, ``"generic"`` any backend, ``"gpu"`` also matches ``"gpu:<x>"``.
``register_b200_kernels(registry)`` adds, to this registry or to the
reference's own (duck-typed: anything with ``register(KernelInfo-like)``),

* ``b200_block_sparse_matmul`` — pattern ``"ij,jk->ik"``, backend ``"gpu"``,
  sparsity ``"sparse"``, priority 10, signature of
  ``block_sparse_matmul_generic(lhs, rhs, block_shape=None)``;
* ``b200_sparse_einsum`` — pattern ``"*"``, same backend/sparsity,
  priority 10, signature of ``execute_sparse``.

Both accept the reference's numpy relations and, with ``host_result=True``
(the default for the adapters registered into a foreign registry), return a
relation of numpy arrays, so callers written against the reference keep
working unchanged.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any, Callable


@dataclass
class KernelInfo:
    """``kernels/registry.py:27-45``."""

    name: str
    pattern: str
    backend: str
    sparsity: str
    priority: int
    kernel_fn: Callable[..., Any]


def _pattern_matches(registered: str, query: str) -> bool:
    return registered == "*" or registered == query


def _backend_matches(registered: str, query: str) -> bool:
    return registered == "generic" or registered == query or query.startswith(registered + ":")


def _sparsity_matches(registered: str, query: str) -> bool:
    return registered == "any" or registered == query


def _detect_backend() -> str:
    """"gpu" when a CUDA device is visible, else "cpu" (``kernels/registry.py:226-242``)."""
    try:
        import torch
        if torch.cuda.is_available():
            return "gpu"
    except Exception:  # pragma: no cover
        pass
    return "cpu"


class KernelRegistry:
    """Pattern/backend/sparsity dispatch table (``kernels/registry.py:48-223``).

    Built with the B200 kernels registered (the reference registers its
    generic JAX fallbacks here; this package has no CPU fallback).
    """

    def __init__(self, register_builtins: bool = True) -> None:
        self._kernels: list[KernelInfo] = []
        if register_builtins:
            register_b200_kernels(self, host_result=False)

    def register(self, kernel) -> None:
        self._kernels.append(kernel)

    def _find_candidates(self, pattern, backend, sparsity):
        return [k for k in self._kernels if _pattern_matches(k.pattern, pattern)
                and _backend_matches(k.backend, backend) and _sparsity_matches(k.sparsity, sparsity)]

    def lookup_info(self, pattern: str, backend: str | None = None, sparsity: str = "dense") -> KernelInfo:
        backend = backend or _detect_backend()
        c = self._find_candidates(pattern, backend, sparsity)
        if not c:
            raise ValueError(f"No kernel found for pattern={pattern!r}, backend={backend!r}, "
                             f"sparsity={sparsity!r}")
        c.sort(key=lambda k: k.priority, reverse=True)
        return c[0]

    def lookup(self, pattern: str, backend: str | None = None, sparsity: str = "dense"):
        return self.lookup_info(pattern, backend, sparsity).kernel_fn

    def list_kernels(self, pattern=None, backend=None, sparsity=None) -> list:
        r = list(self._kernels)
        if pattern is not None:
            r = [k for k in r if k.pattern == pattern or k.pattern == "*"]
        if backend is not None:
            r = [k for k in r if _backend_matches(k.backend, backend)]
        if sparsity is not None:
            r = [k for k in r if k.sparsity == sparsity or k.sparsity == "any"]
        return r


class _HostRelation:
    """Plain relation of numpy arrays returned to reference-side callers."""

    def __init__(self, coords, values, shape, tile_shape):
        self.coords, self.values, self.shape, self.tile_shape = coords, values, tuple(shape), tuple(tile_shape)

    @property
    def num_tuples(self):
        return self.coords.shape[0]

    @property
    def ndim(self):
        return len(self.shape)


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


def register_b200_kernels(registry, info_cls=None, host_result=True, relation_cls=None, priority=10):
    """Register the B200 kernels into ``registry`` (ours or the reference's).

    ``info_cls``: the registry's KernelInfo class (defaults to this module's);
    ``relation_cls``: class used for host results (e.g. the reference's
    ``SparseTensorRelation``), defaults to a plain numpy-holding relation.
    """
    info_cls = info_cls or KernelInfo
    registry.register(info_cls(name="b200_block_sparse_matmul", pattern="ij,jk->ik", backend="gpu",
                               sparsity="sparse", priority=priority,
                               kernel_fn=make_block_sparse_matmul_kernel(host_result, relation_cls)))
    registry.register(info_cls(name="b200_sparse_einsum", pattern="*", backend="gpu", sparsity="sparse",
                               priority=priority, kernel_fn=make_sparse_einsum_kernel(host_result, relation_cls)))
    return registry
