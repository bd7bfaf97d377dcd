"""einjax_b200 — einjax's sparse tensor-relational einsum path on B200 (sm_100a).

Drop-in for the reference's sparse execution path (``execute_sparse`` and
friends, the kernel registry, the sparse autodiff primitive). Every compute
step runs in ``libeinsparse.so`` (hand-written CUDA, C ABI in
``include/einsparse.h``); there is no CPU fallback.
"""

from ._lib import EinsparseError, EinsparseUnavailable  # noqa: F401
from .autodiff import _reverse_einsum_string, sparse_einsum, sparse_einsum_raw  # noqa: F401
from .cost_model import B200_PROFILE, calibrate, detect_device_type, install_b200_profile  # noqa: F401
from .kernels import (block_sparse_matmul, block_sparse_matmul_generic, coordinate_join_hash,  # noqa: F401
                      coordinate_join_sorted)
from .partition import tile_shape_to_partition_spec  # noqa: F401
from .plan import PlanStep, execute_sparse_plan, plan_from_path, reduction_keys  # noqa: F401
from .registry import register_b200_kernels  # noqa: F401
from .sparse import (DUPLICATE_POLICIES, SparseTensor, SparseTensorRelation, as_device_tensor,  # noqa: F401
                     check_device_errors, coalesce_coo, compute_sparsity_stats_coo, compute_sparsity_stats_dense,
                     factor_tile_shapes, find_all_factors, tile_coo, tile_dense)
from .sparse_dispatch import (_add_batch_dim, _compute_output_coords, _infer_output_tile_shape,  # noqa: F401
                              _partition_matched_pairs, coordinate_join, execute_sharded_sparse, execute_sparse,
                              kernel_einsum, plan_pairs, segment_sum, tile_einsum)

__version__ = "0.1.0"
