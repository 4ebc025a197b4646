from rusteeze_b200.config.config import (Config, ModelSection, ServerSection, EngineSection,  # noqa: F401
                                         LoggingSection, MetricsSection, SchedulingSection,
                                         SpeculativeSection, QuantizationConfig, config_from_dict)
from rusteeze_b200.config.loader import ConfigLoader, load_config, env_overrides  # noqa: F401
from rusteeze_b200.config.validation import validate_config  # noqa: F401
