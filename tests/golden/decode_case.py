"""Tiny seeded models for the end-to-end decode parity fixtures.

Both the fixture generator (which runs the reference's ``ddtree_generate``
on CPU) and the GPU test (which runs this package's) build the models here:
a Qwen3 target from ``transformers`` and a DFlash draft (the reference's
class in the generator, this package's in the test).  Every parameter is
then overwritten from one seeded generator in sorted-name order, so the two
sides hold identical weights without storing them; a SHA-256 of the
weights is stored to catch drift.

head_dim is 128, the only head size of the attention kernels.  The models
run in float32: the CPU reference and the GPU path then agree to ~1e-6, and
the fixtures are chosen so that every decision (target argmax along the
accepted path, top-k membership, heap order) has a margin above 1e-4.
"""
from __future__ import annotations

import hashlib

import torch

HEAD_DIM = 128


def target_config(vocab: int):
    from transformers import Qwen3Config
    return Qwen3Config(vocab_size=vocab, hidden_size=96, intermediate_size=192, num_hidden_layers=3,
                       num_attention_heads=4, num_key_value_heads=2, head_dim=HEAD_DIM, max_position_embeddings=512,
                       rms_norm_eps=1e-6, rope_theta=10000.0, tie_word_embeddings=False)


def draft_config(vocab: int, block_size: int, mask_token_id: int):
    from transformers import Qwen3Config
    cfg = Qwen3Config(vocab_size=vocab, hidden_size=96, intermediate_size=192, num_hidden_layers=2,
                      num_attention_heads=4, num_key_value_heads=2, head_dim=HEAD_DIM, max_position_embeddings=512,
                      rms_norm_eps=1e-6, rope_theta=10000.0, tie_word_embeddings=False)
    cfg.block_size = block_size
    cfg.num_target_layers = 3
    cfg.dflash_config = {"target_layer_ids": [0, 2], "mask_token_id": mask_token_id}
    return cfg


def seeded_init(model: torch.nn.Module, seed: int, scale: float = 0.15) -> str:
    """Overwrite every parameter from one generator (sorted names): norm
    weights 1 + 0.1 N(0,1), biases 0, everything else scale * N(0,1).
    Returns the SHA-256 of the weights."""
    g = torch.Generator().manual_seed(seed)
    h = hashlib.sha256()
    with torch.no_grad():
        for name, p in sorted(model.named_parameters(), key=lambda kv: kv[0]):
            if name.endswith("norm.weight"):
                val = 1.0 + 0.1 * torch.randn(p.shape, generator=g)
            elif name.endswith(".bias"):
                val = torch.zeros(p.shape)
            else:
                val = scale * torch.randn(p.shape, generator=g)
            p.copy_(val.to(p.dtype))
            h.update(name.encode())
            h.update(val.to(torch.float32).numpy().tobytes())
    return h.hexdigest()


def prompt(seed: int, length: int, vocab: int, exclude: int) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    ids = torch.randint(0, vocab - 1, (1, length), generator=g)
    ids[ids >= exclude] += 1          # never the mask token
    return ids


# (name, vocab, block_size, node budget, prompt length, max_new_tokens); the
# model seed of each case is chosen by the generator and stored with it
CASES = [
    ("v16_b8_t32", 16, 8, 32, 24, 40),
    ("v300_b6_t12", 300, 6, 12, 20, 30),
    ("v64_b16_t20", 64, 16, 20, 33, 32),
]
