"""Helpers shared by evaluation code (reference utils/functions.py:17-73)."""
from __future__ import annotations

from dataclasses import fields
from typing import Any, Optional


def dict_view(obj: Any) -> dict[str, Any]:
    """Field name -> value of a dataclass instance, without copying the values."""
    return {f.name: getattr(obj, f.name) for f in fields(obj)}


def last_boxed_only_string(text: str) -> Optional[str]:
    """Content of the last ``\\boxed{...}`` (or ``\\fbox{...}``) in ``text``, braces balanced.

    Returns None when there is no such command or its braces never close.
    """
    start = text.rfind("\\boxed")
    if start < 0:
        start = text.rfind("\\fbox")
        if start < 0:
            return None
    open_at = text.find("{", start)
    if open_at < 0:
        return None
    depth = 0
    for i in range(open_at, len(text)):
        ch = text[i]
        if ch == "{":
            depth += 1
        elif ch == "}":
            depth -= 1
            if depth == 0:
                return text[open_at + 1:i].strip()
    return None


def compute_benchmark_micro_macro_avg(stats: dict[str, dict[str, float]]) -> dict[str, float]:
    """Per-subset accuracy / invalid rate plus their unweighted means over subsets."""
    out: dict[str, float] = {}
    accs, invalids = [], []
    for name, s in stats.items():
        n = max(1, s["n"])
        out[f"n_{name}"] = s["n"]
        out[f"acc_{name}"] = s["correct"] / n
        out[f"invalid_{name}"] = s["invalid"] / n
        accs.append(out[f"acc_{name}"])
        invalids.append(out[f"invalid_{name}"])
    k = max(1, len(stats))
    out["n"] = len(stats)
    out["acc"] = sum(accs) / k
    out["invalid"] = sum(invalids) / k
    return out
