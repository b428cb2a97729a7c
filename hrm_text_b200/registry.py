"""String-identified classes: ``"module.path@ClassName"``.

The config tree names models as ``baselines.hrm_nocarry_bp_warmup@HierarchicalReasoningModel``
and heads as ``lm_head@LMHead``, resolved relative to a package prefix (``models.`` in the
reference, utils/functions.py:7-14). Here the default prefix is this framework's ``models``
package; evaluation engines and benchmarks use ``hrm_text_b200.evaluation.``-style prefixes.
"""
from __future__ import annotations

import importlib
import inspect

MODELS_PREFIX = "hrm_text_b200.models."


def load_model_class(identifier: str, prefix: str = MODELS_PREFIX):
    module_path, class_name = identifier.split("@")
    module = importlib.import_module(prefix + module_path)
    return getattr(module, class_name)


def get_model_source_path(identifier: str, prefix: str = MODELS_PREFIX):
    module_path, _ = identifier.split("@")
    module = importlib.import_module(prefix + module_path)
    return inspect.getsourcefile(module)
