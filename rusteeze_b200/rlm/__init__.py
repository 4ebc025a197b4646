"""Recursive Language Model (RLM): host orchestration over the engine."""
from rusteeze_b200.rlm.recursive_engine import (EngineInferenceModel, InferenceResult, MockInferenceModel,  # noqa: F401
                                                RecursiveEngine, RLMConfig, RLMResponse)
from rusteeze_b200.rlm.prompt_env import PromptEnvironment, adaptive_chunk, parse_model_output  # noqa: F401
from rusteeze_b200.rlm.recursive_scheduler import RecursiveScheduler, SchedulerLimits  # noqa: F401
from rusteeze_b200.rlm.variable_store import VariableStore  # noqa: F401
