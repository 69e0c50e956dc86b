"""Import-compatible alias of the reference package name.

Code written against mthcom/innerq imports ``innerq.cache``, ``innerq.quant``
and ``innerq.models`` (``src/innerq/__init__.py``).  With this directory on
the import path those imports resolve, unchanged, to the B200 modules of
``innerq_b200``: ``innerq.cache`` IS ``innerq_b200.cache`` (same module
object), and likewise for ``quant``, ``models`` and the two model modules.
The reference's ``lm_eval_innerq_wrapper`` (its lm-eval harness glue) is not
part of this package.
"""
import importlib
import sys

_ALIASES = {
    "cache": "innerq_b200.cache",
    "quant": "innerq_b200.quant",
    "models": "innerq_b200.models",
    "models.llama_innerq": "innerq_b200.models.llama_innerq",
    "models.mistral_innerq": "innerq_b200.models.mistral_innerq",
}

for _name, _target in _ALIASES.items():
    _mod = importlib.import_module(_target)
    sys.modules[f"{__name__}.{_name}"] = _mod
    if "." not in _name:
        globals()[_name] = _mod

__all__ = ["cache", "quant", "models"]
