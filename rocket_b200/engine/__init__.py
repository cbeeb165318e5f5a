from .engine import LLMEngine, StepStats
from .scheduler import Request, Scheduler, Status

__all__ = ["LLMEngine", "StepStats", "Request", "Scheduler", "Status"]
