"""dsv4_plugin.core — expert bank (host pool + HBM slot cache) and offload engine."""

from dsv4_plugin.core.engine import ExpertOffloadEngine, get_engine, is_expert_weight, parse_expert_name

__all__ = ["ExpertOffloadEngine", "get_engine", "is_expert_weight", "parse_expert_name"]
