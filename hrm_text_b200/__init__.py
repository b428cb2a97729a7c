"""HRM-Text on Blackwell: a B200-native (sm_100a) pretraining framework for the HRM-Text
model family (hierarchical H/L recurrent Transformers with PrefixLM packing).

Public entry points:
* ``hrm_text_b200.Trainer`` — build + train (sharded engine, CUDA-graph steps);
* ``hrm_text_b200.config`` — ``PretrainConfig`` and the Hydra-compatible composer;
* ``hrm_text_b200.runtime.factory.build_model`` — model construction from an arch config.
"""
__version__ = "0.1.0"


def __getattr__(name):
    if name == "Trainer":
        from .runtime.trainer import Trainer
        return Trainer
    raise AttributeError(name)
