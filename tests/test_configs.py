"""CPU checks of the workload table, seeded inputs and the byte model."""
import torch

from kernelproblems_b200 import configs as cf


def test_shard_rows_partition():
    for total in (0, 1, 7, 8192, 128256, 131072):
        for world in (1, 2, 3, 4, 8):
            parts = [cf.shard_rows(total, world, r) for r in range(world)]
            assert parts[0].lo == 0 and parts[-1].hi == total
            assert all(a.hi == b.lo for a, b in zip(parts, parts[1:]))
            assert max(p.n for p in parts) - min(p.n for p in parts) <= 1


def test_embedding_ids_distribution():
    c = cf.C2
    ids = cf.embedding_ids(c)
    assert ids.shape == (8, 4096) and ids.dtype == torch.int64
    assert int(ids.min()) >= 0 and int(ids.max()) < c.vocab
    counts = torch.bincount(ids.reshape(-1), minlength=c.vocab)
    top = counts.topk(100).values.sum().item()
    assert top >= 0.05 * c.T  # the hot set carries >= 5% of the tokens
    assert torch.equal(ids, cf.embedding_ids(c)), "seeded"


def test_bytes_match_the_documented_table():
    assert cf.bytes_rmsnorm_fwd(8192, 4096) == 134_258_688
    assert cf.bytes_rmsnorm_bwd(8192, 4096) == 201_383_936
    assert cf.bytes_embedding_fwd(32768, 4096) == 537_133_056
    assert cf.bytes_embedding_bwd(32768, 4096, 128256) == 2_370_043_904
    assert cf.bytes_rope(32768, 32, 8, 128) == 671_350_784
    assert cf.bytes_add_rmsnorm_fwd(131072, 8192, rstd=False) == 8_589_950_976
    assert cf.bytes_add_rmsnorm_bwd(131072, 8192) == 8_590_508_032


def test_weight_distribution():
    w = cf.rmsnorm_weight(4096).float()
    assert abs(w.mean().item() - 1.0) < 0.01 and abs(w.std().item() - 0.1) < 0.01
