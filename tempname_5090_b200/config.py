"""Model / run configuration: the reference's defaults and the B200 benchmark config.

`REFERENCE_DEFAULT` mirrors TempName-5090's DEFAULT_CONFIG
(python/flux_5090/model.py:13-15); `GPT_6P7B_BENCH` is the benchmark config
(micro-batch 4, vocab 50304, AdamW lr 1e-4).  Both give 8192 tokens per step.
Validation rules follow model.py:20-47 and parameter counting model.py:50-59,
extended to TP size 1 (the reference requires W >= 2 for its operator only).
"""
from __future__ import annotations

import math

REFERENCE_DEFAULT = dict(layers=32, hidden=4096, ffn=16384, heads=32, sequence=2048,
                         micro_batch=1, accumulation_steps=4, vocab=33792, chunk_rows=128)
GPT_6P7B_BENCH = dict(layers=32, hidden=4096, ffn=16384, heads=32, sequence=2048,
                      micro_batch=4, accumulation_steps=1, vocab=50304, chunk_rows=128)
SMALL = dict(layers=2, hidden=256, ffn=1024, heads=4, sequence=256, micro_batch=2,
             accumulation_steps=1, vocab=1024, chunk_rows=128)
ARMS = ("flux", "flux_taco", "flux_taco_interleaved", "flux_taco_interleaved_arrival")
INTEGER_KEYS = tuple(REFERENCE_DEFAULT)
FLOAT_KEYS = (("learning_rate", 1e-4), ("weight_decay", 0.01), ("max_grad_norm", 1.0),
              ("layer_norm_epsilon", 1e-5))


def validate_config(config: dict, world_size: int = 8) -> dict:
    """Return a completed, validated copy of `config` for TP size `world_size`."""
    if not isinstance(config, dict):
        raise ValueError("model config must be a dictionary")
    result = dict(REFERENCE_DEFAULT)
    result.update(config)
    for name in INTEGER_KEYS:
        if type(result[name]) is not int or result[name] <= 0:
            raise ValueError(f"{name} must be a positive integer")
    if type(world_size) is not int or world_size < 1:
        raise ValueError("world_size must be a positive integer")
    for name in ("hidden", "ffn", "heads", "vocab"):
        if result[name] % world_size:
            raise ValueError(f"{name} must be divisible by tensor-parallel size")
    if result["hidden"] % result["heads"]:
        raise ValueError("hidden must be divisible by heads")
    rows = result["sequence"] * result["micro_batch"]
    if rows % world_size or (rows // world_size) % result["chunk_rows"]:
        raise ValueError("sequence rows per rank must be divisible by chunk_rows")
    for key, default in FLOAT_KEYS:
        value = result.get(key, default)
        if isinstance(value, bool) or not isinstance(value, (int, float)) or not math.isfinite(value):
            raise ValueError(f"{key} must be finite")
        if value < 0 or (key in ("learning_rate", "max_grad_norm", "layer_norm_epsilon") and value == 0):
            raise ValueError(f"invalid {key}")
        result[key] = float(value)
    return result


def parameter_counts(config: dict, world_size: int = 8) -> dict:
    c = validate_config(config, world_size)
    h, f, v, s, layers = (c[k] for k in ("hidden", "ffn", "vocab", "sequence", "layers"))
    logical = v * h + s * h + layers * (4 * h * h + 2 * h * f + 9 * h + f) + 2 * h
    replicated = s * h + layers * 6 * h + 2 * h
    sharded = logical - replicated
    return dict(logical_parameters=logical, replicated_parameters=replicated,
                sharded_parameters=sharded,
                parameters_per_rank=sharded // world_size + replicated,
                tied_embedding_head=True)


def train_flops_per_step(config: dict) -> float:
    """Model FLOPs of one optimizer step (forward + backward, causal attention)."""
    c = validate_config(config, 1)
    h, f, v, s, L = (c[k] for k in ("hidden", "ffn", "vocab", "sequence", "layers"))
    tokens = s * c["micro_batch"] * c["accumulation_steps"]
    dense = 2 * tokens * (L * (4 * h * h + 2 * h * f) + v * h)
    attention = 2 * 2 * tokens * s * h * L / 2  # QK^T and PV, causal half
    return 3.0 * (dense + attention)
