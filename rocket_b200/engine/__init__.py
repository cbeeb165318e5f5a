from .drafts import AdaptiveChain, Chain, DraftModel, DraftSource, make_draft_source
from .engine import Detached, EngineFaulted, LLMEngine, SchedulerStall, StepStats
from .scheduler import Request, Scheduler, Status

__all__ = ["EngineFaulted", "SchedulerStall", "LLMEngine", "StepStats", "Detached", "Request", "Scheduler", "Status",
           "DraftSource", "DraftModel", "Chain", "AdaptiveChain", "make_draft_source"]
