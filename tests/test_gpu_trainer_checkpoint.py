"""Checkpoint / resume of the data-parallel GPT-2 trainer: a trainer restored
from another trainer's checkpoint takes the same next step (same loss, same
fp32 master weights after AdamW) as the original."""

import pytest
import torch

from nexar_b200.models.gpt2 import GPT2Config
from nexar_b200.parallel.dp import DataParallelTrainer

pytestmark = pytest.mark.gpu

def _batch(cfg, seed):
    g = torch.Generator().manual_seed(seed)
    idx = torch.randint(0, cfg.vocab_size, (2, cfg.block_size), generator=g)
    tgt = torch.randint(0, cfg.vocab_size, (2, cfg.block_size), generator=g)
    return idx, tgt


def test_resume_matches_uninterrupted_run(cuda0, tmp_path):
    cfg = GPT2Config.tiny()
    a = DataParallelTrainer(cfg, micro_batch=2, seq_len=cfg.block_size, use_cuda_graph=False, seed=0)
    for s in range(2):
        a.step(*_batch(cfg, s))
    path = str(tmp_path / "dp.pt")
    a.save(path)
    b = DataParallelTrainer(cfg, micro_batch=2, seq_len=cfg.block_size, use_cuda_graph=False, seed=1)
    assert not torch.equal(a.model.flat.master, b.model.flat.master)  # different initialisation
    b.load(path)
    torch.testing.assert_close(b.model.flat.master, a.model.flat.master, rtol=0, atol=0)
    assert int(b.step_dev.item()) == 2
    la = a.step(*_batch(cfg, 7))
    lb = b.step(*_batch(cfg, 7))
    assert abs(la - lb) <= 1e-4 * max(1.0, abs(la)), (la, lb)
    # The step after the restore matches up to the order of atomic additions
    # (the embedding and LayerNorm backward kernels add with atomics, so the
    # last bits of a gradient can differ between runs; one AdamW step turns
    # that into differences far below one update of lr = 6e-4).
    torch.testing.assert_close(b.model.flat.master, a.model.flat.master, rtol=1e-3, atol=5e-5)

    other = GPT2Config(n_layer=1, n_head=4, n_embd=128, vocab_size=1000, padded_vocab=1024, block_size=64)
    c = DataParallelTrainer(other, micro_batch=2, seq_len=other.block_size, use_cuda_graph=False)
    with pytest.raises(ValueError, match="model"):
        c.load(path)
