"""Pretraining / SFT driver (the ``pretrain.py`` entry point; reference pretrain.py:167-388).

    python pretrain.py [--config-name cfg_sft] [group@pkg=option] [key=value] [+key=value]
    torchrun --nproc_per_node=8 pretrain.py arch/size@arch=L lr=2.5e-4 global_batch_size=172032

Flow per rank: process group (NCCL on GPU, gloo on CPU) when launched by torchrun; config
composed on rank 0 and broadcast; seed ``seed + rank``; the PrefixLM dataset with the
multipack sampler in a persistent DataLoader worker; the model built on the device and
wrapped by the sharded engine (CUDA-graph steps on GPU); optional resume; then epochs of
``train_step`` with the warm-up + cosine learning rate and the bp-steps warm-up, metrics
reduced to rank 0 every ``log_interval`` steps, and a checkpoint every
``checkpoint_interval`` epochs (and after the last).
"""
from __future__ import annotations

import math
import os
import sys
from dataclasses import dataclass
from datetime import timedelta
from pathlib import Path
from typing import Optional

import torch
import torch.distributed as dist
from torch.utils.data import DataLoader

from ..config import PretrainConfig, compose, parse_cli
from ..data.dataset import V1Dataset, V1DatasetConfig
from ..registry import get_model_source_path
from ..utils.logging import MetricLogger
from . import checkpoint as ckpt
from .factory import build_model, model_config_dict
from .perf import ThroughputMeter, step_flops
from .trainer import Trainer
from .watchdog import Heartbeat, StepWatchdog
from ..utils.errors import check_device_errors


@dataclass
class TrainState:
    step: int
    total_steps: int


def lr_at(config: PretrainConfig, step: int, total_steps: int) -> float:
    """Linear warm-up, then cosine decay to ``lr * lr_min_ratio`` (pretrain.py:191-203)."""
    if step < config.lr_warmup_steps:
        return config.lr * min(1.0, step / max(1, config.lr_warmup_steps))
    span = max(1, total_steps - config.lr_warmup_steps)
    progress = (step - config.lr_warmup_steps) / span
    cosine = max(0.0, (1 - config.lr_min_ratio) * 0.5 * (1.0 + math.cos(math.pi * progress)))
    return config.lr * (config.lr_min_ratio + cosine)


def init_distributed():
    """Returns ``(world, rank, local_rank, device)``; initialises a process group under torchrun."""
    if "LOCAL_RANK" not in os.environ:
        device = torch.device("cuda", 0) if torch.cuda.is_available() else torch.device("cpu")
        if device.type == "cuda":
            torch.cuda.set_device(device)
        return 1, 0, 0, device
    local = int(os.environ["LOCAL_RANK"])
    # collectives that wait longer than this fail instead of hanging (a rank that left the job)
    timeout = timedelta(seconds=float(os.environ.get("HRM_PG_TIMEOUT_S", "1800")))
    if torch.cuda.is_available():
        device = torch.device("cuda", local)
        torch.cuda.set_device(device)
        dist.init_process_group("nccl", device_id=device, timeout=timeout)
    else:
        device = torch.device("cpu")
        dist.init_process_group("gloo", timeout=timeout)
    return dist.get_world_size(), dist.get_rank(), local, device


def load_synced_config(config_name: str, overrides: list[str], rank: int) -> PretrainConfig:
    objects = [None]
    if rank == 0:
        config = PretrainConfig(**compose(config_name, overrides))
        if config.project_name is None:
            config.project_name = f"{Path(config.data.path).stem.capitalize()} HLM-torch"
        if config.run_name is None:
            config.run_name = os.environ.get("MLP_TASK_NAME", f"{config.arch.name.split('@')[-1]} {os.getpid()}")
        if config.checkpoint_path is None:
            config.checkpoint_path = os.path.join("checkpoints", config.project_name, config.run_name)
        objects = [config]
    if dist.is_initialized():
        dist.broadcast_object_list(objects, src=0)
    return objects[0]


def create_dataloader(config: PretrainConfig, local_batch: int, rank: int, world: int, num_workers: int = 1):
    dataset = V1Dataset(V1DatasetConfig(seed=config.seed, dataset_path=config.data.path,
                                        drop_last_batch=True, target_only=config.data.target_only,
                                        batch_max_length=local_batch, rank=rank, num_replicas=world))
    loader = DataLoader(dataset, batch_size=None, num_workers=num_workers,
                        prefetch_factor=8 if num_workers > 0 else None, pin_memory=torch.cuda.is_available(),
                        persistent_workers=num_workers > 0)
    return loader, dataset.metadata


def reduce_metrics(metrics: dict, prefix: str, rank: int) -> Optional[dict]:
    """Sum ``(numerator, denominator)`` pairs on rank 0 and divide (pretrain.py:215-224)."""
    keys = sorted(metrics)
    values = torch.stack([metrics[k][0].float() for k in keys] + [metrics[k][1].float() for k in keys])
    if dist.is_initialized():
        dist.reduce(values, dst=0)
    if rank != 0:
        return None
    num, den = values.chunk(2)
    out = (num / den.clamp_min(1e-12)).cpu().tolist()
    return {prefix + k: v for k, v in zip(keys, out)}


def run(config_name: str, overrides: list[str], max_steps: Optional[int] = None, num_workers: int = 1) -> dict:
    world, rank, local, device = init_distributed()
    config = load_synced_config(config_name, overrides, rank)
    torch.random.manual_seed(config.seed + rank)

    assert config.global_batch_size % world == 0, "global_batch_size must be divisible by the world size"
    local_batch = config.global_batch_size // world
    loader, metadata = create_dataloader(config, local_batch, rank, world, num_workers)
    model_cfg = model_config_dict(config.arch.model_dump(), metadata.model_dump(), config.data.model_dump())

    model = build_model(model_cfg, device)
    if dist.is_initialized():
        for buf in model.buffers():
            dist.broadcast(buf, src=0)
    trainer = Trainer(model_cfg, beta1=config.beta1, beta2=config.beta2, weight_decay=config.weight_decay,
                      ema=config.ema, device=device, model=model)
    total_steps = int(config.epochs * metadata.total_length // config.global_batch_size)
    state = TrainState(step=0, total_steps=total_steps)

    if config.resume_from is not None:
        epoch = ckpt.load_checkpoint(trainer.params, model, config.resume_from, config.resume_epoch,
                                     betas=(config.beta1, config.beta2), weight_decay=config.weight_decay,
                                     ema=config.ema, weights_only_from_ema=config.weights_only_resume_from_ema)
        if rank == 0:
            print(f"[Resume] loaded epoch {epoch} from {config.resume_from}")

    logger = MetricLogger(config, enabled=rank == 0, total_steps=total_steps)
    if rank == 0:
        logger.log({"num_params": sum(s.numel for s in trainer.params.slots)}, step=0)
        if config.checkpoint_path is not None:
            ckpt.write_run_files(config.checkpoint_path, config.model_dump(), metadata.model_dump(),
                                 get_model_source_path(config.arch.name))

    # Failure detection (off unless asked for): a per-step deadline that reports and
    # interrupts a stuck rank, and a store heartbeat checked before each logging collective.
    deadline = float(os.environ.get("HRM_STEP_DEADLINE_S", "0"))
    watchdog = StepWatchdog(deadline) if deadline > 0 else None
    heartbeat = None
    if dist.is_initialized() and os.environ.get("HRM_HEARTBEAT", "0") == "1":
        heartbeat = Heartbeat(dist.distributed_c10d._get_default_store(), rank, world)

    meter = ThroughputMeter(device, world)
    last, lr = {}, 0.0
    for epoch in range(1, config.epochs + 1):
        for batch, _info in loader:
            state.step += 1
            lr = lr_at(config, state.step, total_steps)
            extra = model.compute_train_extra_args(state)
            if watchdog is not None:
                watchdog.arm(state.step)
            flops = step_flops(model, batch, extra)
            _loss, metrics = trainer.train_step_async(batch, lr, extra.get("bp_steps"))
            meter.step(local_batch * world, flops)
            if heartbeat is not None:
                heartbeat.set_step(state.step)
            if state.step % config.log_interval == 0:
                if watchdog is not None and device.type == "cuda":
                    check_device_errors()  # a device wait that gave up fails the step here
                if heartbeat is not None:
                    stale = heartbeat.stale_ranks(max_age_s=max(30.0, deadline))
                    if stale:
                        raise RuntimeError(f"ranks {stale} stopped heart-beating; aborting before the next collective")
                reduced = reduce_metrics(metrics, "train/", rank)
                perf = meter.report()
                if rank == 0:
                    last = reduced | extra | {"train/lr": lr} | perf
                    logger.log(last, step=state.step)
            if max_steps is not None and state.step >= max_steps:
                break
        if (epoch % config.checkpoint_interval == 0 or epoch == config.epochs) and config.checkpoint_path:
            ckpt.save_checkpoint(trainer.params, model, config.checkpoint_path, epoch, carry=None, lr=lr, rank=rank)
        if max_steps is not None and state.step >= max_steps:
            break

    if watchdog is not None:
        watchdog.close()
    if heartbeat is not None:
        heartbeat.stop()
    trainer.close()
    logger.finish()
    if dist.is_initialized():
        dist.destroy_process_group()
    return last


def main(argv: Optional[list[str]] = None) -> None:
    config_name, overrides = parse_cli(sys.argv[1:] if argv is None else argv)
    max_steps = os.environ.get("HRM_MAX_STEPS")
    run(config_name, overrides, max_steps=int(max_steps) if max_steps else None)
