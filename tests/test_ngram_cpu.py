"""Hashed n-gram input embedding: bucket hashing, mean combine, gradients, and a grug model with it."""

import torch

from marin_experiments_b200.config import GrugModelConfig, NgramEmbedConfig, dumps, loads
from marin_experiments_b200.models.grug import Transformer
from marin_experiments_b200.ops import reference as R


def test_buckets_depend_on_the_ngram_only():
    a = torch.tensor([[5, 6, 7, 8, 9]])
    b = torch.tensor([[1, 6, 7, 8, 2]])
    ba, bb = R.ngram_buckets(a, 2, 0, 1000), R.ngram_buckets(b, 2, 0, 1000)
    assert ba[0, 2] == bb[0, 2] and ba[0, 3] == bb[0, 3]  # same bigrams (6,7), (7,8)
    assert ba[0, 1] != bb[0, 1] or ba[0, 4] != bb[0, 4]
    assert not torch.equal(R.ngram_buckets(a, 2, 0, 1000), R.ngram_buckets(a, 2, 1, 1000))
    assert int(ba.max()) < 1000 and int(ba.min()) >= 0


def test_embed_mean_and_grad():
    table = torch.randn(2, 50, 8, requires_grad=True)
    ids = torch.randint(0, 30, (2, 7))
    out = R.ngram_embed(ids, table, (2, 3), 2)
    assert out.shape == (14, 8)
    out.sum().backward()
    assert torch.isclose(table.grad.sum(), torch.tensor(14 * 8.0))  # each row's 4 lookups average to 1


def test_model_with_ngram():
    ng = NgramEmbedConfig(orders=(2, 3), num_hashes=2, hash_buckets=997, rank=16)
    cfg = GrugModelConfig(vocab_size=256, hidden_dim=64, intermediate_dim=128, shared_expert_intermediate_dim=128,
                          num_experts=4, num_experts_per_token=2, num_layers=2, num_heads=2, num_kv_heads=2,
                          head_dim=32, max_seq_len=32, sliding_window=32, ngram=ng)
    assert loads(dumps(cfg)).ngram == ng
    m = Transformer(cfg).init_weights(0)
    tok = torch.randint(0, 256, (2, 32))
    loss, _ = m.next_token_loss(tok)
    loss.backward()
    assert m.ngram_table.grad is not None and m.ngram_table.grad.abs().sum() > 0
    assert m.ngram_proj.grad.abs().sum() > 0
