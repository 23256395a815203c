"""Serving this framework's Llama runtime over an OpenAI-compatible API:
a continuous-batching engine (:mod:`.engine`), its HTTP front (:mod:`.api`),
the server CLI (``python -m connex_b200.serve``) and the downstream pipeline
stage CLI (``python -m connex_b200.serve.stage``)."""
from connex_b200.serve.engine import (EngineFull, GenerationEngine, ModelStepper, PipelineStepper, Request,
                                      RuleStepper, Stepper)

__all__ = ["EngineFull", "GenerationEngine", "ModelStepper", "PipelineStepper", "Request", "RuleStepper",
           "Stepper"]
