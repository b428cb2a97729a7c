"""Generation engines for the evaluation harness (reference evaluation/engines.py).

* ``SimpleEngine`` — this framework's checkpoint + continuous-batching generator;
* ``VLLMEngine`` — vLLM for Hugging Face checkpoints (e.g. an exported HRM-Text model or a
  baseline LM).
"""
from __future__ import annotations

from typing import Optional


class BaseEngine:
    def generate(self, prompts: list[str], **kwargs) -> list[str]:
        raise NotImplementedError


class VLLMEngine(BaseEngine):
    def __init__(self, ckpt_path: str, **kwargs):
        from vllm import LLM
        self.llm = LLM(model=ckpt_path, **kwargs)

    def generate(self, prompts: list[str], temperature: float = 0.0, max_tokens: Optional[int] = None,
                 stop=None) -> list[str]:
        from vllm import SamplingParams
        outs = self.llm.generate(prompts, SamplingParams(temperature=temperature, max_tokens=max_tokens, stop=stop))
        return [o.outputs[0].text for o in outs]


class SimpleEngine(BaseEngine):
    def __init__(self, ckpt_path: str, ckpt_epoch: Optional[int] = None, ckpt_use_ema: bool = True):
        from hrm_text_b200.inference.engine import inference_load_checkpoint
        self.ckpt = inference_load_checkpoint(ckpt_path, ckpt_epoch, ckpt_use_ema)

    def generate(self, prompts: list[str], batch_size: int = 100, max_context: int = 1024,
                 max_tokens: Optional[int] = None, temperature: float = 0.0, condition: str = "direct") -> list[str]:
        from hrm_text_b200.inference.engine import inference_generate
        max_tokens = max_context if max_tokens is None else max_tokens
        outputs = [""] * len(prompts)
        work = iter([(i, (condition, p.strip())) for i, p in enumerate(prompts)])
        try:
            from tqdm import tqdm
            bar = tqdm(total=len(prompts), desc="generation")
        except Exception:
            bar = None
        for pid, text in inference_generate(self.ckpt, work, max_context, max_tokens, batch_size, temperature):
            outputs[pid] = text
            if bar is not None:
                bar.update()
        if bar is not None:
            bar.close()
        return outputs
