"""Exporters producing dli.graph.v1 graphs + dli.weights.v1 payloads for the sm_100a plugin."""
from .qwen2 import (QWEN2_0_5B, QWEN2_7B, QWEN2_72B, Qwen2Shape, build_graph, export_qwen2,
                    random_state, rotary_tables, transform_weights, write_weights)

__all__ = ["Qwen2Shape", "QWEN2_0_5B", "QWEN2_7B", "QWEN2_72B", "build_graph", "export_qwen2",
           "random_state", "rotary_tables", "transform_weights", "write_weights"]
