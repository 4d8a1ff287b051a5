"""`EngineConfig` under the reference's module path
(afterimage/runtime/config.py): the same class as
afterimage_b200.runtime.streaming_engine.EngineConfig."""
from .streaming_engine import EngineConfig

__all__ = ["EngineConfig"]
