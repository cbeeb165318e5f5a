from .context import ParallelCtx, init_from_env

__all__ = ["ParallelCtx", "init_from_env"]
