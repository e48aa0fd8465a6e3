"""Temperature sampling (``ddt_sample_rows``), the temperature > 0 branch of
sample(logits, temperature) (model/utils.py:31-35).

The reference draws with torch.multinomial from softmax(logits / T); the
kernel draws from the same distribution with its own generator, so parity is
checked on distributions: each token's frequency over many independent rows
must lie within 5 standard errors of its softmax probability (float64),
tokens of probability 0 are never drawn, and the same (seed, offset) repeats
the draws exactly."""
import ctypes

import numpy as np
import pytest
import torch


def _k():
    from ddtree_eagle3_patch_b200 import kernels
    return kernels


def _softmax64(logits, t):
    z = np.asarray(logits, np.float64) / t
    z = z - z[np.isfinite(z)].max()
    p = np.exp(z)
    return p / p.sum()


def _check_freq(draws, p, n):
    counts = np.bincount(draws, minlength=len(p)).astype(np.float64)
    f = counts / n
    se = np.sqrt(p * (1 - p) / n)
    assert np.all(np.abs(f - p) <= 5 * se + 1e-12), np.c_[f, p, se][np.abs(f - p) > 5 * se]
    assert counts[p == 0].sum() == 0


def test_validation_without_gpu():
    from ddtree_eagle3_patch_b200 import _lib
    lib = _lib.load()
    assert lib.ddt_sample_rows(None, 0, 4, 10, 10, 0.0, 1, 0, None, None, 0, None) == 1   # temperature 0
    assert b"temperature" in lib.ddt_last_error()
    assert lib.ddt_sample_rows(None, 0, 4, 10, 10, float("inf"), 1, 0, None, None, 0, None) == 1
    assert lib.ddt_sample_rows(None, 0, 4, 10, 5, 1.0, 1, 0, None, None, 0, None) == 1      # row_stride < vocab
    assert lib.ddt_sample_rows(None, 0, 0, 10, 10, 1.0, 1, 0, None, None, 0, None) == 0     # no rows: nothing to do
    assert lib.ddt_sample_rows_workspace_size(65, 151936) >= 65 * 16 * 8


@pytest.mark.gpu
@pytest.mark.parametrize("dtype,t", [(torch.float32, 0.7), (torch.bfloat16, 1.0), (torch.float16, 2.5)])
def test_small_vocab_frequencies(dtype, t):
    K = _k()
    base = torch.tensor([0.0, 0.5, 1.0, 1.5, -1.0, 2.0, float("-inf"), 0.3, -3.0])
    base = base.to(dtype).float()              # the values the kernel sees
    n = 40000
    x = base.to(dtype).cuda().expand(n, -1).contiguous()
    draws = K.sample_rows(x, t, seed=1234).cpu().numpy()
    _check_freq(draws, _softmax64(base.numpy(), t), n)


@pytest.mark.gpu
def test_large_vocab_mass_across_chunks():
    """Vocab 151936 (chunks of 9496 tokens): five heavy tokens in different
    chunks plus the rest, as one 'other' bucket."""
    K = _k()
    V, n, t = 151936, 3000, 1.0
    g = torch.Generator().manual_seed(5)
    base = torch.randn(V, generator=g) * 0.5
    heavy = [3, 9496 * 2 + 1, 9496 * 7 + 4, 100000, V - 1]
    base[heavy] = torch.tensor([9.0, 9.5, 8.5, 10.0, 9.2])
    base = base.to(torch.bfloat16)
    p = _softmax64(base.float().numpy(), t)
    x = base.cuda().expand(n, -1).contiguous()
    draws = K.sample_rows(x, t, seed=77, offset=3).cpu().numpy()
    bucket = np.full(V, len(heavy), np.int64)
    bucket[heavy] = np.arange(len(heavy))
    pb = np.array([p[h] for h in heavy] + [1.0 - p[heavy].sum()])
    _check_freq(bucket[draws], pb, n)


@pytest.mark.gpu
def test_same_seed_repeats_and_offset_changes():
    K = _k()
    x = torch.randn(65, 151936, device="cuda").to(torch.bfloat16)
    a = K.sample_rows(x, 1.0, seed=9, offset=0)
    b = K.sample_rows(x, 1.0, seed=9, offset=0)
    c = K.sample_rows(x, 1.0, seed=9, offset=1)
    d = K.sample_rows(x, 1.0, seed=10, offset=0)
    assert torch.equal(a, b)
    assert not torch.equal(a, c) and not torch.equal(a, d)
    assert int(a.min()) >= 0 and int(a.max()) < 151936


@pytest.mark.gpu
def test_tiny_temperature_is_argmax_and_sample_mirror():
    K = _k()
    g = torch.Generator().manual_seed(2)
    x = torch.randn(65, 151936, generator=g)
    idx = torch.randint(0, 151936, (65,), generator=g)
    x[torch.arange(65), idx] += 12.0            # a clear maximum per row
    x = x.cuda()
    assert torch.equal(K.sample_rows(x, 1e-3, seed=4).cpu(), idx)
    assert torch.equal(K.sample(x, 0.0).cpu(), idx)                # greedy branch
    torch.manual_seed(123)
    s1 = K.sample(x[None], 1.0)
    torch.manual_seed(123)
    s2 = K.sample(x[None], 1.0)
    assert s1.shape == (1, 65) and torch.equal(s1, s2)


@pytest.mark.gpu
def test_eagle3_posterior_at_temperature_matches_reference_distribution():
    """evaluate_eagle3_posterior at T > 0 (eagle3.py:46-79): every verify row
    draws once from softmax(logits / T), the accepted length is the longest
    matching prefix of the path, and the bonus token is a second draw from
    the last accepted row.  On a three-node path with P(row 0 -> a) = 0.6
    and P(row 1 -> b) = 0.5, the lengths 0 / 1 / 2 come out with
    probabilities 0.4 / 0.3 / 0.3, and after length 0 the bonus token follows
    row 0's distribution; both within 5 standard errors over 4000 calls."""
    from ddtree_eagle3_patch_b200.eagle3 import evaluate_eagle3_posterior
    dev = torch.device("cuda", 0)
    V, t = 8, 0.7
    a, b = 3, 5
    p0 = np.full(V, 0.4 / (V - 1))
    p0[a] = 0.6
    p1 = np.full(V, 0.5 / (V - 1))
    p1[b] = 0.5
    p2 = np.full(V, 1.0 / V)
    logits = torch.tensor(np.log(np.stack([p0, p1, p2])) * t, dtype=torch.float32, device=dev)[None]
    draft = torch.tensor([[1, a, b]], dtype=torch.long, device=dev)
    retrieve = torch.tensor([[0, 1, 2]], dtype=torch.long, device=dev)
    torch.manual_seed(123)
    n = 4000
    lengths, bonus0 = np.zeros(3, np.int64), []
    for _ in range(n):
        best, length, tok, cand, acc = evaluate_eagle3_posterior(logits, draft, retrieve, t)
        assert best == 0 and acc == [0, 1, 2][: length + 1]
        lengths[length] += 1
        if length == 0:
            bonus0.append(int(tok.item()))
    expect = np.array([0.4, 0.3, 0.3])
    se = np.sqrt(expect * (1 - expect) / n)
    assert np.all(np.abs(lengths / n - expect) <= 5 * se), lengths
    m = len(bonus0)
    freq = np.bincount(bonus0, minlength=V) / m
    assert np.all(np.abs(freq - p0) <= 5 * np.sqrt(p0 * (1 - p0) / m) + 1e-12), freq
