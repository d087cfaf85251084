"""Execution driver (reference ``worker/executor.py``)."""

from .executor import ExecutionMetrics, LayerTiming, ParallelExecutor

__all__ = ["ExecutionMetrics", "LayerTiming", "ParallelExecutor"]
