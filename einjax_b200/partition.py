"""Tile shape -> partition spec; mirrors einjax ``sharding/partition.py``.

A dimension whose tile is smaller than the tensor is tiled ("upper case") and
gets a mesh axis name; a dimension held whole ("lower case") gets None
(``sharding/partition.py:17-92``). In this package the device split itself
is done by ``einjax_b200.distributed`` over output tiles or over the
contracted tile range; this function keeps the reference's metadata contract
and its ValueError rules for callers that use it.
"""

from __future__ import annotations


def tile_shape_to_partition_spec(shape, tile_shape, mesh_axis_names=("x", "y", "z", "w")) -> tuple:
    if len(shape) != len(tile_shape):
        raise ValueError(f"shape ({len(shape)}D) and tile_shape ({len(tile_shape)}D) must have the same "
                         f"number of dimensions")
    for d, (s, t) in enumerate(zip(shape, tile_shape)):
        if t > s:
            raise ValueError(f"tile_shape[{d}]={t} exceeds shape[{d}]={s}")
        if t <= 0:
            raise ValueError(f"tile_shape[{d}]={t} must be positive")
        if s % t != 0:
            raise ValueError(f"shape[{d}]={s} is not evenly divisible by tile_shape[{d}]={t}")
    tiled = [t != s for s, t in zip(shape, tile_shape)]
    if sum(tiled) > len(mesh_axis_names):
        raise ValueError(f"Need {sum(tiled)} mesh axes for sharded dimensions but only "
                         f"{len(mesh_axis_names)} axis names available: {mesh_axis_names}")
    spec, axis = [], 0
    for t in tiled:
        if t:
            spec.append(mesh_axis_names[axis])
            axis += 1
        else:
            spec.append(None)
    return tuple(spec)
