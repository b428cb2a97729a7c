"""Inference entry points under the reference's module name (simple_inference_engine.py).

``inference_load_checkpoint(ckpt_path, ckpt_epoch, ckpt_use_ema)`` and
``inference_generate(ckpt, iterator, max_tokens, max_generation, batch_size, temp)``; see
``hrm_text_b200.inference.engine``.
"""
from hrm_text_b200.inference.engine import (InferenceCheckpoint, generate_tokens, inference_generate,  # noqa: F401
                                            inference_load_checkpoint, load_model_from_checkpoint, sample)
