"""Training configuration: schema plus a small Hydra-compatible composer.

The schema mirrors the reference's ``PretrainConfig`` / ``ArchConfig`` / ``DataConfig``
(pretrain.py:33-79): same field names, types and defaults, so an ``all_config.yaml``
written by either framework loads in the other.

Hydra and OmegaConf are not part of this framework's dependencies. ``compose`` implements
the subset of Hydra's composition that the config tree uses:

* a ``defaults`` list of ``group@package: option`` entries plus ``_self_``
  (config/cfg_pretrain.yaml), where ``arch/net@arch: hrm`` merges ``config/arch/net/hrm.yaml``
  into the ``arch`` node;
* command-line overrides ``group@package=option`` (choose another option of a group),
  ``a.b=value`` (override an existing key), ``+a.b=value`` (add a key) and
  ``++a.b=value`` (add or override);
* ``???`` marks a mandatory value that must be set by an override.

Values are parsed as YAML scalars, as Hydra does (``lr=2.5e-4`` is a float,
``ema=null`` is None, ``run_only=[A,B]`` is a list).
"""
from __future__ import annotations

import copy
import os
from typing import Any, Optional, Sequence

import pydantic
import yaml

MISSING = "???"

CONFIG_DIR = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "config")


class ArchConfig(pydantic.BaseModel):
    """Model selection; every other key is architecture-specific and passes through."""

    model_config = pydantic.ConfigDict(extra="allow")

    name: str
    head: str


class DataConfig(pydantic.BaseModel):
    model_config = pydantic.ConfigDict(extra="allow")

    path: str
    target_only: bool = True  # supervise the response only


class PretrainConfig(pydantic.BaseModel):
    arch: ArchConfig
    data: DataConfig

    global_batch_size: int
    epochs: int

    lr: float
    lr_min_ratio: float
    lr_warmup_steps: int

    weight_decay: float
    beta1: float
    beta2: float
    ema: Optional[float] = None
    fwd_bwd_dtype: str = "bfloat16"

    project_name: Optional[str] = None
    run_name: Optional[str] = None
    checkpoint_path: Optional[str] = None

    resume_from: Optional[str] = None
    resume_epoch: Optional[int] = None
    weights_only_resume_from_ema: bool = False

    seed: int = 0
    checkpoint_interval: int = 1
    log_interval: int = 5


# ----------------------------------------------------------------------------------------
# composition
# ----------------------------------------------------------------------------------------

def _load_yaml(path: str) -> dict:
    with open(path, "r") as f:
        data = yaml.safe_load(f)
    return data if data is not None else {}


def _merge(dst: dict, src: dict) -> dict:
    """Recursive dict merge; values of ``src`` win."""
    for key, value in src.items():
        if isinstance(value, dict) and isinstance(dst.get(key), dict):
            _merge(dst[key], value)
        else:
            dst[key] = copy.deepcopy(value)
    return dst


def _set_path(tree: dict, dotted: str, value: Any, *, must_exist: bool, may_exist: bool = True) -> None:
    keys = dotted.split(".")
    node = tree
    for key in keys[:-1]:
        if key not in node or not isinstance(node[key], dict):
            if must_exist:
                raise KeyError(f"Could not override '{dotted}': key '{key}' is not in the config. "
                               f"Use '+{dotted}=...' to add it.")
            node[key] = {}
        node = node[key]
    if must_exist and keys[-1] not in node:
        raise KeyError(f"Could not override '{dotted}': key is not in the config. Use '+{dotted}=...' to add it.")
    if not may_exist and keys[-1] in node:
        raise KeyError(f"Could not append '{dotted}': key already exists. Use '++{dotted}=...' to force.")
    node[keys[-1]] = value


def _parse_value(text: str) -> Any:
    if text == "":
        return ""
    try:
        return yaml.safe_load(text)
    except yaml.YAMLError:
        return text


def _check_missing(tree: Any, prefix: str = "") -> None:
    if isinstance(tree, dict):
        for key, value in tree.items():
            _check_missing(value, f"{prefix}{key}.")
    elif tree == MISSING:
        raise ValueError(f"Missing mandatory value: {prefix[:-1]}")


def _parse_default(entry: Any) -> tuple[Optional[str], Optional[str], Optional[str]]:
    """``{"arch/net@arch": "hrm"}`` -> (group, package, option); ``"_self_"`` -> (None, None, None)."""
    if isinstance(entry, str):
        if entry == "_self_":
            return None, None, None
        # bare config name in the same directory is not used by this tree
        raise ValueError(f"Unsupported defaults entry: {entry!r}")
    (key, option), = entry.items()
    group, _, package = key.partition("@")
    return group, (package or group.replace("/", ".")), option


def compose(config_name: str = "cfg_pretrain", overrides: Sequence[str] = (), config_dir: str = CONFIG_DIR) -> dict:
    """Compose ``config_dir/<config_name>.yaml`` with Hydra-style ``overrides`` into a plain dict."""
    primary = _load_yaml(os.path.join(config_dir, f"{config_name}.yaml"))
    defaults = primary.pop("defaults", ["_self_"])
    primary.pop("hydra", None)

    group_choice: dict[tuple[str, str], Optional[str]] = {}
    order: list[Optional[tuple[str, str]]] = []
    for entry in defaults:
        group, package, option = _parse_default(entry)
        if group is None:
            order.append(None)
        else:
            group_choice[(group, package)] = option
            order.append((group, package))

    value_overrides: list[tuple[str, str, Any]] = []
    for ov in overrides:
        if "=" not in ov:
            raise ValueError(f"Override must be key=value: {ov!r}")
        lhs, rhs = ov.split("=", 1)
        if "/" in lhs.lstrip("+"):  # group choice: arch/size@arch=L
            group, _, package = lhs.lstrip("+").partition("@")
            package = package or group.replace("/", ".")
            if (group, package) not in group_choice:
                order.append((group, package))
            group_choice[(group, package)] = rhs
            continue
        if lhs.startswith("++"):
            value_overrides.append(("force", lhs[2:], _parse_value(rhs)))
        elif lhs.startswith("+"):
            value_overrides.append(("add", lhs[1:], _parse_value(rhs)))
        else:
            value_overrides.append(("set", lhs, _parse_value(rhs)))

    tree: dict = {}
    for item in order:
        if item is None:
            _merge(tree, primary)
            continue
        group, package = item
        option = group_choice[item]
        if option is None or option == "null":
            continue
        data = _load_yaml(os.path.join(config_dir, group, f"{option}.yaml"))
        node = tree
        for key in package.split(".") if package else []:
            node = node.setdefault(key, {})
        _merge(node, data)

    for kind, path, value in value_overrides:
        if kind == "set":
            _set_path(tree, path, value, must_exist=True)
        elif kind == "add":
            _set_path(tree, path, value, must_exist=False, may_exist=False)
        else:
            _set_path(tree, path, value, must_exist=False)

    _check_missing(tree)
    return tree


def parse_cli(argv: Sequence[str]) -> tuple[str, list[str]]:
    """Split ``--config-name X`` / ``--config-name=X`` from the override list."""
    config_name, overrides = "cfg_pretrain", []
    it = iter(range(len(argv)))
    skip = False
    for i in it:
        if skip:
            skip = False
            continue
        arg = argv[i]
        if arg in ("--config-name", "-cn"):
            config_name = argv[i + 1]
            skip = True
        elif arg.startswith("--config-name="):
            config_name = arg.split("=", 1)[1]
        else:
            overrides.append(arg)
    return config_name, overrides


def load_pretrain_config(config_name: str = "cfg_pretrain", overrides: Sequence[str] = ()) -> PretrainConfig:
    return PretrainConfig(**compose(config_name, overrides))
