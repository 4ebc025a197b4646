"""rusteeze_b200: a Blackwell (sm_100a) native LLM inference engine.

Layers (bottom to top):
  core/       request/response/sampling types and errors
  ops/        hand-written sm_100a CUDA kernels and their fp32 PyTorch oracles
  models/     model zoo (Llama, Mistral, Mixtral, Qwen2, Phi3, Gemma/Gemma2)
  parallel/   one-process-per-GPU tensor/expert parallelism over NCCL and NVLink peer memory
  engine/     continuous-batching scheduler, paged KV block manager, model runner, sampler
  tokenizer/  HF tokenizers, chat templates, incremental detokenizer
  rlm/        Recursive Language Model orchestration over the engine
  api/        OpenAI-compatible HTTP server
  metrics/    Prometheus registry, structured logging, NVTX tracing
  config/     typed configuration (defaults < file < env < CLI)
  cli/        `rusteeze` command line
"""

__version__ = "0.1.0"

from rusteeze_b200.core.sampling_params import SamplingParams  # noqa: E402,F401
from rusteeze_b200.core.outputs import RequestOutput, CompletionOutput  # noqa: E402,F401


def __getattr__(name):
    # Heavy imports (torch models, engine) are resolved lazily so that
    # `import rusteeze_b200` stays cheap for the CLI and API layers.
    if name in ("LLM", "LLMEngine"):
        from rusteeze_b200.engine import llm_engine
        return getattr(llm_engine, name)
    raise AttributeError(name)
