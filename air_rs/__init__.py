"""air_rs — a B200-native (sm_100a) LLM inference engine with Air.rs's public surface.

    >>> import air_rs
    >>> engine = air_rs.load("model.gguf")
    >>> print(engine.generate("Hello"))
"""
from __future__ import annotations

import asyncio
import os
from concurrent.futures import ThreadPoolExecutor
from typing import AsyncGenerator

__version__ = "1.3.0"

from . import utils  # noqa: E402
from .api import Engine, GenerateConfig, GbnfConstraint, Metrics, TokenChannel  # noqa: E402

_STREAM_EXECUTOR: ThreadPoolExecutor | None = None


def _get_executor() -> ThreadPoolExecutor:
    global _STREAM_EXECUTOR
    if _STREAM_EXECUTOR is None:
        _STREAM_EXECUTOR = ThreadPoolExecutor(max_workers=4, thread_name_prefix="air_rs_stream")
    return _STREAM_EXECUTOR


async def astream(engine: Engine, prompt: str, config: GenerateConfig | None = None, *,
                  executor: ThreadPoolExecutor | None = None) -> AsyncGenerator[str, None]:
    """Async generator yielding decoded tokens as they are produced.

    Generation runs on a worker thread; each ``recv_sync`` wait runs in the executor so the
    event loop is never blocked.
    """
    pool = executor or _get_executor()
    loop = asyncio.get_running_loop()
    channel = await loop.run_in_executor(pool, lambda: engine._stream_channel(prompt, config))
    while True:
        token = await loop.run_in_executor(pool, channel.recv_sync)
        if token is None:
            return
        yield token


def shutdown_stream_executor(wait: bool = True) -> None:
    """Shut down the shared streaming thread pool (safe to call repeatedly)."""
    global _STREAM_EXECUTOR
    if _STREAM_EXECUTOR is not None:
        _STREAM_EXECUTOR.shutdown(wait=wait)
        _STREAM_EXECUTOR = None


def load(target: str, **kwargs) -> Engine:
    """Load an Engine from a GGUF path or a model-registry alias (offline cache only)."""
    if not os.path.exists(target):
        from .hub import resolve
        target = resolve(target)
    return Engine.from_gguf(target, **kwargs)


__all__ = ["Engine", "GenerateConfig", "GbnfConstraint", "Metrics", "TokenChannel", "astream", "load",
           "shutdown_stream_executor", "utils", "__version__"]
