"""Host-side mirror of the Ferrite Strata plugin interface, for driving
libstrata_b200.so from Python (tests, benchmarks, integration)."""
from .ir import (BF16, E2M1, E4M3, E8M0, F32, I32, W4G32, DType, Graph, GraphBuilder, Op, encode_graph, frame,
                 shape_class, w8pc)
from .plugin import BoundRun, Buffer, Device, Executable, Plugin, PluginLoadError, StrataError

__all__ = ["BF16", "E2M1", "E4M3", "E8M0", "F32", "I32", "W4G32", "DType", "Graph", "GraphBuilder", "Op", "encode_graph",
           "frame", "shape_class", "w8pc", "BoundRun", "Buffer", "Device", "Executable", "Plugin",
           "PluginLoadError", "StrataError"]
