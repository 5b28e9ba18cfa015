"""GPT forward/backward and a training step on the GPU vs the CPU oracle run
of the same parameters (same model code, torch reference math on CPU)."""
import pytest
import torch

pytestmark = pytest.mark.gpu

CFG = dict(layers=2, hidden=256, ffn=1024, heads=2, sequence=512, micro_batch=2,
           accumulation_steps=1, vocab=2048, chunk_rows=128)


def rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-12)).item()


def test_gpu_model_matches_cpu_oracle():
    from tempname_5090_b200.models.gpt import GPT
    from tempname_5090_b200._native import check_status
    gpu = GPT(CFG, device="cuda", seed=3)
    cpu = GPT(CFG, device="cpu", seed=3, init=False)
    cpu.load_state_dict({k: v.cpu() for k, v in gpu.state_dict().items()})
    g = torch.Generator().manual_seed(1)
    M = CFG["sequence"] * CFG["micro_batch"]
    tokens = torch.randint(0, CFG["vocab"], (M,), generator=g)
    targets = torch.randint(0, CFG["vocab"], (M,), generator=g)
    lg = gpu.forward_backward(tokens.cuda(), targets.cuda())
    lc = cpu.forward_backward(tokens, targets)
    torch.cuda.synchronize()
    check_status()
    assert abs(lg.item() - lc.item()) < 1e-2 * abs(lc.item())
    for name in gpu.state_dict():
        assert rel(gpu.g[name].cpu(), cpu.g[name]) < 5e-2, name


def test_training_reduces_loss_and_is_deterministic():
    from tempname_5090_b200.models.gpt import GPT
    from tempname_5090_b200.models.train import Trainer
    losses = []
    finals = []
    for _ in range(2):
        model = GPT(CFG, device="cuda", seed=5)
        trainer = Trainer(model, lr=3e-3)
        g = torch.Generator().manual_seed(2)
        M = CFG["sequence"] * CFG["micro_batch"]
        tokens = torch.randint(0, 64, (M,), generator=g)
        labels = (tokens + 1) % 64
        run = []
        for _ in range(8):
            loss, norm = trainer.train_step([(tokens.pin_memory(), labels.pin_memory())])
            run.append(loss)
        losses.append(run)
        finals.append(model.store.flat.clone())
    assert losses[0][-1] < losses[0][0] - 0.5
    assert losses[0] == losses[1]
    assert torch.equal(finals[0], finals[1])


def test_state_dict_roundtrip_gpu(tmp_path):
    from tempname_5090_b200.models.gpt import GPT
    from tempname_5090_b200.utils.checkpoint import save_checkpoint, load_checkpoint
    from tempname_5090_b200.models.train import Trainer
    model = GPT(CFG, device="cuda", seed=9)
    trainer = Trainer(model)
    g = torch.Generator().manual_seed(4)
    M = CFG["sequence"] * CFG["micro_batch"]
    batch = [(torch.randint(0, CFG["vocab"], (M,), generator=g), torch.randint(0, CFG["vocab"], (M,), generator=g))]
    trainer.train_step(batch)
    save_checkpoint(str(tmp_path), model, trainer)
    model2 = GPT(CFG, device="cuda", seed=99)
    trainer2 = Trainer(model2)
    load_checkpoint(str(tmp_path), model2, trainer2)
    a = trainer.train_step(batch)
    b = trainer2.train_step(batch)
    assert a == b
