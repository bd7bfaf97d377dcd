"""Inert sharding placeholders for the golden-vector generator."""

import numpy as _np


class Mesh:
    def __init__(self, devices, axis_names):
        self.devices = _np.asarray(devices, dtype=object)
        self.axis_names = tuple(axis_names)


class PartitionSpec(tuple):
    def __new__(cls, *parts):
        return super().__new__(cls, parts)


class NamedSharding:
    def __init__(self, mesh, spec):
        self.mesh, self.spec = mesh, spec
