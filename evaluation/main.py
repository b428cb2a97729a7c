"""Benchmark runner (reference evaluation/main.py).

    python -m evaluation.main ckpt_path=checkpoints/... [config=evaluation/config/hrm_benchmarking.yaml]
        [run_only=[MATH,DROP]] [generation_config.batch_size=16]

The YAML config names an engine (``engines@<Engine>``) and a list of benchmarks
(``benchmarks@<Benchmark>``); command-line ``key=value`` pairs are merged over it (dotted
keys address nested fields). Benchmarks that share the same final generation settings are
generated in one batch, then each benchmark scores its slice.
"""
from __future__ import annotations

import json
import sys
from collections import defaultdict
from typing import Any, Optional

import pydantic
import yaml

from hrm_text_b200.config import _merge, _parse_value, _set_path
from hrm_text_b200.registry import load_model_class


class BenchmarkConfig(pydantic.BaseModel):
    model_config = pydantic.ConfigDict(extra="allow")
    name: str
    generation_config: dict[str, Any] = {}


class EvaluationConfig(pydantic.BaseModel):
    model_config = pydantic.ConfigDict(extra="allow")
    run_only: Optional[list[str]] = None
    engine: str
    generation_config: dict[str, Any] = {}
    benchmarks: list[BenchmarkConfig]

    @pydantic.model_validator(mode="after")
    def _check_run_only(self):
        if self.run_only is not None:
            assert self.run_only, "run_only cannot be empty"
            known = {b.name for b in self.benchmarks}
            unknown = [n for n in self.run_only if n not in known]
            if unknown:
                raise ValueError(f"Unknown benchmark name in run_only: {unknown}")
        return self


def load_config(argv: list[str]) -> EvaluationConfig:
    cli = {}
    for arg in argv:
        key, _, value = arg.partition("=")
        _set_path(cli, key.lstrip("+"), _parse_value(value), must_exist=False)
    path = cli.pop("config", "evaluation/config/hrm_benchmarking.yaml")
    with open(path) as f:
        base = yaml.safe_load(f)
    return EvaluationConfig(**_merge(base, cli))


def run(cfg: EvaluationConfig, engine=None) -> dict:
    if engine is None:
        print(f"Initializing Engine: {cfg.engine}...")
        engine = load_model_class(f"engines@{cfg.engine}", prefix="evaluation.")(**(cfg.__pydantic_extra__ or {}))
    groups: dict[str, dict] = defaultdict(lambda: {"prompts": [], "benchmarks": []})
    for b_cfg in cfg.benchmarks:
        if cfg.run_only is not None and b_cfg.name not in cfg.run_only:
            continue
        bench = load_model_class(f"benchmarks@{b_cfg.name}", prefix="evaluation.")(**(b_cfg.__pydantic_extra__ or {}))
        gen = cfg.generation_config | bench.generation_overrides | b_cfg.generation_config
        key = json.dumps(gen, sort_keys=True)
        start = len(groups[key]["prompts"])
        groups[key]["prompts"].extend(bench.prompts)
        groups[key]["benchmarks"].append((b_cfg.name, bench, start, len(groups[key]["prompts"])))
    results = {}
    for key, group in groups.items():
        gen = json.loads(key)
        template = gen.pop("prompt_template", "{prompt}")
        prompts = [template.format(prompt=p) for p in group["prompts"]]
        print(f"Running generation batch of {len(prompts)} prompts with {gen}")
        outputs = engine.generate(prompts, **gen)
        for name, bench, s, e in group["benchmarks"]:
            results[name] = bench.compute_metrics(outputs[s:e])
    print("\n" + "#" * 50 + "\nEVALUATION SUMMARY\n" + "#" * 50)
    for name, metrics in results.items():
        print(f"\n--- {name} ---")
        for k, v in metrics.items():
            print(f"{k:.<25}: {v:.4f}" if isinstance(v, float) else f"{k:.<25}: {v}")
    return results


def main(argv: Optional[list[str]] = None) -> None:
    run(load_config(sys.argv[1:] if argv is None else argv))


if __name__ == "__main__":
    main()
