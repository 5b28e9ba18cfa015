"""TP-sharded checkpoint save / resume.

One file per rank, `rank{r}-of-{W}.pt`, holding the rank's parameters under
the reference state_dict names (python/flux_5090/model.py:206-229 of
TempName-5090: embedding, position, layers.i.*, final_*) plus, when a trainer
is given, the FP32 master weights and AdamW moments in the same named layout
and the step counter.  Writes are atomic (temporary file + rename).  Loading
checks the TP size, the configuration and every name and shape.
"""
from __future__ import annotations

import json
import os

import torch


def _file(directory: str, rank: int, world: int) -> str:
    return os.path.join(directory, f"rank{rank}-of-{world}.pt")


def _named_region(model, flat: torch.Tensor) -> dict:
    st = model.store
    out = {}
    for s in st.specs:
        o = st.offsets[s.name]
        out[s.name] = flat[o:o + s.numel].view(s.shape)
    return out


def save_checkpoint(directory: str, model, trainer=None) -> str:
    os.makedirs(directory, exist_ok=True)
    payload = dict(format="tempname-5090-b200-tp-checkpoint-v1", world=model.world, rank=model.rank,
                   config=json.loads(json.dumps(model.config)), arm=model.arm,
                   params={k: v.detach().cpu().clone() for k, v in model.state_dict().items()})
    if trainer is not None:
        payload["optimizer"] = dict(
            step=trainer.step_count,
            master={k: v.cpu().clone() for k, v in _named_region(model, trainer.master).items()},
            exp_avg={k: v.cpu().clone() for k, v in _named_region(model, trainer.m).items()},
            exp_avg_sq={k: v.cpu().clone() for k, v in _named_region(model, trainer.v).items()})
    path = _file(directory, model.rank, model.world)
    tmp = path + ".tmp"
    torch.save(payload, tmp)
    os.replace(tmp, path)
    return path


def load_checkpoint(directory: str, model, trainer=None) -> dict:
    path = _file(directory, model.rank, model.world)
    payload = torch.load(path, map_location="cpu", weights_only=False)
    if payload.get("format") != "tempname-5090-b200-tp-checkpoint-v1":
        raise ValueError("not a tempname-5090-b200 checkpoint")
    if payload["world"] != model.world or payload["rank"] != model.rank:
        raise ValueError("checkpoint TP size/rank differs from the model")
    if payload["config"] != json.loads(json.dumps(model.config)):
        raise ValueError("checkpoint configuration differs from the model")
    model.load_state_dict(payload["params"])
    if trainer is not None:
        opt = payload.get("optimizer")
        if opt is None:
            raise ValueError("checkpoint has no optimizer state")
        for field, target in (("master", trainer.master), ("exp_avg", trainer.m), ("exp_avg_sq", trainer.v)):
            views = _named_region(model, target)
            for name, t in opt[field].items():
                views[name].copy_(t)
        trainer.step_count = int(opt["step"])
    return payload
