"""Token selection on vocabulary shards and the embedding exchange, against
the oracle (src/layers/sampler.py:4-17, src/layers/llm_head.py:38-69).

* greedy: the selected token is torch.argmax of the full row (lowest index on
  ties), bit-exact, whatever the sharding of the vocabulary;
* sampling with given Exp(1) draws: the reference sampler's token
  (softmax(l / T) / E, argmax) on the same draws;
* sampling with the in-kernel Philox draws: independent of the sharding
  (draws are keyed by global column) and distributed as softmax(l / T);
* the embedding exchange at world 1 equals the lookup kernel bit for bit.
Multi-rank exchanges run in tests/test_tp_gpu.py.
"""
import pytest
import torch

from oracle import layers as L

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _logits(B, V, seed, scale=3.0):
    g = torch.Generator().manual_seed(seed)
    x = (torch.randn(B, V, generator=g) * scale).to(torch.bfloat16)
    # planted ties: two equal maxima per row, the lower index must win
    for b in range(0, B, 3):
        j = int(torch.randint(0, V - 1, (1,), generator=g))
        k = int(torch.randint(j + 1, V, (1,), generator=g))
        x[b, j] = x[b, k] = x[b].max() + 1
    return x


def _sharded_keys(logits, shards, **kw):
    from src import b200
    V = logits.shape[1]
    bounds = [V * i // shards for i in range(shards + 1)]
    keys = []
    for i in range(shards):
        part = logits[:, bounds[i]:bounds[i + 1]]
        nz = kw.get("noise")
        kwi = dict(kw)
        if nz is not None:
            kwi["noise"] = nz[:, bounds[i]:bounds[i + 1]].contiguous()
        keys.append(b200.select_tokens(part.contiguous(), bounds[i], **kwi))
    return torch.stack(keys).max(0).values


@pytest.mark.parametrize("B,V", [(1, 7), (5, 1000), (256, 151936), (64, 18992)])
def test_greedy_selection_is_torch_argmax(B, V):
    from src import b200
    x = _logits(B, V, seed=V)
    want = x.float().argmax(-1)
    for shards in (1, 2, 3, 8):
        if shards > V:
            continue
        keys = _sharded_keys(x.to(DEV), shards)
        got = b200.tokens_from_keys(keys)
        torch.cuda.synchronize()
        assert torch.equal(got.cpu(), want), shards
    assert torch.equal(b200.argmax(x.to(DEV)).cpu(), want)


@pytest.mark.parametrize("B,V", [(8, 1000), (256, 151936)])
def test_sampling_with_given_draws_matches_oracle_sampler(B, V):
    from src import b200
    from src.layers.sampler import Sampler
    x = _logits(B, V, seed=3 * V, scale=2.0)
    g = torch.Generator().manual_seed(7)
    temps = (torch.rand(B, generator=g) * 1.5 + 0.1).float()
    noise = torch.empty(B, V).exponential_(1, generator=g)
    want = L.sample(x, temps, noise)
    got = Sampler(seed=1)(x.to(DEV), temps.to(DEV), noise=noise.to(DEV))
    for shards in (2, 8):
        keys = _sharded_keys(x.to(DEV), shards, temperatures=temps.to(DEV), noise=noise.to(DEV))
        assert torch.equal(b200.tokens_from_keys(keys).cpu(), want), shards
    torch.cuda.synchronize()
    assert torch.equal(got.cpu(), want)


def test_philox_sampling_is_shard_independent_and_follows_softmax():
    from src import b200
    # shard independence on a full-size row
    x = _logits(16, 151936, seed=5, scale=1.0)
    temps = torch.full((16,), 0.8)
    one = b200.tokens_from_keys(b200.select_tokens(x.to(DEV), 0, temps.to(DEV), seed=11, offset=3))
    for shards in (2, 4, 8):
        keys = _sharded_keys(x.to(DEV), shards, temperatures=temps.to(DEV), seed=11, offset=3)
        assert torch.equal(b200.tokens_from_keys(keys).cpu(), one.cpu()), shards
    # distribution over a small vocabulary: 4096 rows x 1 draw each
    V = 6
    base = torch.tensor([0.0, 1.0, -0.5, 2.0, 0.3, -2.0])
    rows = 4096
    xs = base.repeat(rows, 1).to(torch.bfloat16)
    T = torch.full((rows,), 1.3)
    counts = torch.zeros(V)
    for off in range(4):
        tok = b200.tokens_from_keys(b200.select_tokens(xs.to(DEV), 0, T.to(DEV), seed=99, offset=off))
        counts += torch.bincount(tok.cpu(), minlength=V).float()
    n = counts.sum()
    p = torch.softmax(xs[0].float() / 1.3, -1)
    # multinomial standard error per category, 5 sigma
    assert ((counts / n - p).abs() <= 5 * (p * (1 - p) / n).sqrt() + 1e-3).all(), (counts / n, p)


def test_embedding_exchange_world1_is_the_lookup():
    from src import b200
    g = torch.Generator().manual_seed(2)
    V, H, T = 5000, 1024, 300
    w = torch.randn(V, H, generator=g).to(torch.bfloat16).to(DEV)
    ids = torch.randint(-3, V + 3, (T,), generator=g).to(DEV)  # a few ids outside the table
    want = b200.embedding(ids, w, 0, V)
    out = torch.full((T, H), 7.0, dtype=torch.bfloat16, device=DEV)
    b200.embedding_exchange(ids, w, 0, V, V, 0, 1, [out.data_ptr()], H, None, None)
    torch.cuda.synchronize()
    assert torch.equal(out, want)
    assert torch.equal(want.cpu(), L.vocab_embedding(ids.cpu(), w.cpu(), 0, V))
