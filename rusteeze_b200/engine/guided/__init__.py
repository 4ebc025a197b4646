"""Guided (structured) decoding: regex automaton, JSON Schema to regex, token masks."""
from rusteeze_b200.engine.guided.guide import Guide, fsm_for, guide_pattern, index_for  # noqa: F401
