from rusteeze_b200.metrics.registry import EngineMetrics, Timer  # noqa: F401
from rusteeze_b200.metrics.logging_setup import init_logging, nvtx_range  # noqa: F401
