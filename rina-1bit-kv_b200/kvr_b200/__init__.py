"""kvr_b200 — B200-native (sm_100a) compressed-KV hot path of KVR
("Key-predicted Value Retrieval"), drop-in for the reference package
``modules`` (modules/__init__.py:3-13)."""

from .kvr_window import WindowBuffer
from .kvr_retrieval import RetrievalIndex

__all__ = ["WindowBuffer", "RetrievalIndex", "KVRHook", "KVRGenerator"]


def __getattr__(name):
    # the model-integration classes pull in transformers; import them lazily
    if name == "KVRHook":
        from .kvr_hook import KVRHook
        return KVRHook
    if name == "KVRGenerator":
        from .kvr_generator import KVRGenerator
        return KVRGenerator
    raise AttributeError(name)
