from .engine import EngineFaulted, LLMEngine, StepStats
from .scheduler import Request, Scheduler, Status

__all__ = ["EngineFaulted", "LLMEngine", "StepStats", "Request", "Scheduler", "Status"]
