from .engine import EngineFaulted, LLMEngine, SchedulerStall, StepStats
from .scheduler import Request, Scheduler, Status

__all__ = ["EngineFaulted", "SchedulerStall", "LLMEngine", "StepStats", "Request", "Scheduler", "Status"]
