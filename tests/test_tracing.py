"""Named trace scopes: absent unless enabled, present in a profiler trace when
enabled (model layers forward/backward, optimizer), exported with a digest."""
import json

import torch


def _tiny():
    from tempname_5090_b200.models.gpt import GPT
    from tempname_5090_b200.models.train import Trainer
    cfg = dict(layers=2, hidden=256, ffn=512, heads=2, sequence=128, micro_batch=2,
               accumulation_steps=1, vocab=512, chunk_rows=128)
    model = GPT(cfg, device="cpu", seed=3)
    g = torch.Generator().manual_seed(1)
    tokens = torch.randint(0, cfg["vocab"], (256,), generator=g)
    return Trainer(model), [(tokens, tokens.roll(1))]


def _names(prof):
    return {e.name for e in prof.events()}


def test_scopes_only_when_enabled(tmp_path):
    from tempname_5090_b200.utils import tracing
    trainer, batches = _tiny()
    acts = [torch.profiler.ProfilerActivity.CPU]
    with torch.profiler.profile(activities=acts) as prof:
        trainer.step(batches)
    assert not any(n.startswith("gpt.layer") for n in _names(prof))
    assert not tracing.is_enabled()
    with tracing.enabled(), torch.profiler.profile(activities=acts) as prof:
        trainer.step(batches)
    names = _names(prof)
    for want in ("gpt.layer0.forward", "gpt.layer1.forward", "gpt.layer1.backward", "gpt.layer0.backward",
                 "trainer.micro_batch0", "trainer.optimizer"):
        assert want in names, want
    assert not tracing.is_enabled()
    path, sha = tracing.export(prof, tmp_path / "t" / "trace.json")
    data = json.loads(open(path).read())
    assert any(e.get("name") == "trainer.optimizer" for e in data["traceEvents"])
    import hashlib
    assert sha == hashlib.sha256(open(path, "rb").read()).hexdigest()
