"""Training-metric logging: Weights & Biases when available (and not disabled), else stdout.

Metric keys match the reference (``train/loss``, ``train/accuracy``, ``train/exact_accuracy``,
``train/lr``, ``bp_steps``, ``num_params``; reference pretrain.py:344-370). wandb system stats
are disabled as in the reference.
"""
from __future__ import annotations

import json
import os
import sys


class MetricLogger:
    def __init__(self, config, enabled: bool, total_steps: int = 0):
        self.enabled = enabled
        self._wandb = None
        self._bar = None
        if not enabled:
            return
        if os.environ.get("WANDB_MODE", "") != "disabled":
            try:
                import wandb
                wandb.init(project=config.project_name, name=config.run_name, config=config.model_dump(),
                           settings=wandb.Settings(_disable_stats=True))
                self._wandb = wandb
            except Exception as exc:  # no credentials / offline: fall back to stdout
                print(f"[log] wandb unavailable ({type(exc).__name__}); logging to stdout", file=sys.stderr)
        try:
            import tqdm
            self._bar = tqdm.tqdm(total=total_steps, disable=not sys.stderr.isatty())
        except Exception:
            self._bar = None

    def log(self, metrics: dict, step: int) -> None:
        if not self.enabled:
            return
        if self._bar is not None:
            self._bar.update(step - self._bar.n)
        if self._wandb is not None:
            self._wandb.log(metrics, step=step)
        else:
            print(json.dumps({"step": step} | {k: (float(v) if isinstance(v, (int, float)) else v)
                                               for k, v in metrics.items()}), flush=True)

    def finish(self) -> None:
        if self._bar is not None:
            self._bar.close()
        if self._wandb is not None:
            self._wandb.finish()
