"""Checkpoint / resume on CPU: saving after two optimizer steps and resuming in
a fresh model + trainer continues bitwise like the uninterrupted run; loading
rejects a different configuration, TP size or a missing optimizer state; and
gradient accumulation over micro-batches is exact."""
import pytest
import torch

CFG = dict(layers=2, hidden=256, ffn=512, heads=2, sequence=128, micro_batch=2,
           accumulation_steps=1, vocab=512, chunk_rows=128)


def _batches(seed):
    g = torch.Generator().manual_seed(seed)
    t = torch.randint(0, CFG["vocab"], (256,), generator=g)
    return [(t, torch.roll(t, 1))]


def _trainer(seed=5, cfg=CFG):
    from tempname_5090_b200.models.gpt import GPT
    from tempname_5090_b200.models.train import Trainer
    return Trainer(GPT(cfg, device="cpu", seed=seed))


def test_resume_continues_bitwise(tmp_path):
    from tempname_5090_b200.utils.checkpoint import load_checkpoint, save_checkpoint
    a = _trainer()
    for s in range(2):
        a.step_host(_batches(s))
    save_checkpoint(str(tmp_path), a.model, a)
    b = _trainer(seed=99)  # different initialisation: everything must come from the checkpoint
    load_checkpoint(str(tmp_path), b.model, b)
    assert b.step_count == a.step_count == 2
    la, na = a.step_host(_batches(7))
    lb, nb = b.step_host(_batches(7))
    assert (la, na) == (lb, nb)
    for (ka, va), (kb, vb) in zip(a.model.state_dict().items(), b.model.state_dict().items()):
        assert ka == kb and torch.equal(va, vb), ka
    assert torch.equal(a.master, b.master) and torch.equal(a.m, b.m) and torch.equal(a.v, b.v)


def test_load_rejects_mismatches(tmp_path):
    from tempname_5090_b200.utils.checkpoint import load_checkpoint, save_checkpoint
    a = _trainer()
    save_checkpoint(str(tmp_path / "params_only"), a.model)
    with pytest.raises(ValueError, match="optimizer"):
        load_checkpoint(str(tmp_path / "params_only"), a.model, a)
    save_checkpoint(str(tmp_path / "full"), a.model, a)
    other = _trainer(cfg=dict(CFG, ffn=1024))
    with pytest.raises(ValueError, match="configuration"):
        load_checkpoint(str(tmp_path / "full"), other.model, other)
    (tmp_path / "full" / "rank0-of-1.pt").rename(tmp_path / "full" / "rank0-of-2.pt")
    with pytest.raises(FileNotFoundError):
        load_checkpoint(str(tmp_path / "full"), a.model, a)


def test_gradient_accumulation_matches_single_batch():
    """Two identical micro-batches with accumulation_steps=2 (loss scale 1/2,
    FP32 gradient accumulator) take exactly the step of one batch with
    accumulation_steps=1."""
    one = _trainer(cfg=CFG)
    two = _trainer(cfg=dict(CFG, accumulation_steps=2))
    b = _batches(11)
    for _ in range(2):
        l1, n1 = one.step_host(b)
        l2, n2 = two.step_host(b + b)
        assert (l1, n1) == (l2, n2)
    for (k, v1), (_, v2) in zip(one.model.state_dict().items(), two.model.state_dict().items()):
        assert torch.equal(v1, v2), k
