"""innerq_b200: the InnerQ KV-cache decode hot path on B200 (sm_100a).

Drop-in modules mirroring the reference package ``innerq`` (mthcom/innerq):

* ``innerq_b200.quant``  — ``src/innerq/quant.py``
* ``innerq_b200.cache``  — ``src/innerq/cache.py``
* ``innerq_b200.models`` — ``src/innerq/models`` (Llama / Mistral hooks plus the
  ``"innerq"`` attention function that reads the packed cache directly)

Compute runs in ``libinnerq_b200.so`` (hand-written CUDA for sm_100a, C ABI in
``include/innerq_b200.h``); there is no CPU fallback.
"""
from . import _lib  # noqa: F401

__all__ = ["quant", "cache", "models", "attention", "store"]


def __getattr__(name):
    import importlib
    if name in __all__:
        return importlib.import_module(f".{name}", __name__)
    raise AttributeError(name)
