"""Synthetic task generators: determinism, layout and bit-parity with the reference stream."""
import torch

from exploration_b200 import data


def digest(t):
    weights = torch.arange(1, t.numel() + 1).reshape(t.shape)
    return int((t.long() * weights).sum() % 1000000007)


def test_generator_streams_match_reference_digests():
    # Digests of the reference generators (st/data/synthetic.py) at these seeds.
    g = torch.Generator().manual_seed(1234)
    out = data.mqar_batch(2, 96, g, "cpu", n_pairs=8, n_queries=3, key_tokens=1)
    assert [digest(x) for x in out[:3]] == [534025, 527339, 846]
    g = torch.Generator().manual_seed(99)
    out = data.mqar_batch(2, 200, g, "cpu", n_pairs=10, n_queries=4, key_tokens=2)
    assert [digest(x) for x in out[:3]] == [2530639, 2517269, 2352]
    g = torch.Generator().manual_seed(5)
    out = data.passkey_batch(3, 64, g, "cpu")
    assert [digest(x) for x in out] == [392968, 387013, 1890, 105]
    g = torch.Generator().manual_seed(6)
    out = data.copying_batch(2, 64, g, "cpu")
    assert [digest(x) for x in out[:3]] == [196577, 195957, 1480]


def test_mqar_deterministic_per_seed():
    a = data.mqar_batch(2, 256, torch.Generator().manual_seed(7), "cpu", n_pairs=8, n_queries=2,
                        key_tokens=2)
    b = data.mqar_batch(2, 256, torch.Generator().manual_seed(7), "cpu", n_pairs=8, n_queries=2,
                        key_tokens=2)
    for x, y in zip(a, b):
        assert (x is None and y is None) or torch.equal(x, y)


def test_two_token_keys_unique_and_targets_are_digits():
    idx, tgt, mask, extra = data.mqar_batch(4, 2048, torch.Generator().manual_seed(3), "cpu",
                                            n_pairs=32, n_queries=4, key_tokens=2)
    assert extra is None
    assert bool((mask.sum(1) == 4).all())
    assert bool(((tgt[mask] >= 0) & (tgt[mask] <= 9)).all())
    seq = torch.cat([idx, tgt[:, -1:]], 1)
    for row in seq.tolist():
        keys = {(row[i], row[i + 1]) for i in range(len(row) - 2)
                if 34 <= row[i] <= 97 and 34 <= row[i + 1] <= 97 and 0 <= row[i + 2] <= 9}
        assert len(keys) == 32


def test_query_layout():
    for kt in (1, 2):
        idx, tgt, mask, _ = data.mqar_batch(2, 1024, torch.Generator().manual_seed(5), "cpu",
                                            n_pairs=16, n_queries=4, key_tokens=kt)
        seq = torch.cat([idx, tgt[:, -1:]], 1)
        for row in range(2):
            for j in mask[row].nonzero().flatten().tolist():
                assert seq[row, j - kt].item() == data.Q
                for u in range(kt):
                    assert 34 <= seq[row, j - kt + 1 + u] <= 97


def test_resolve_npairs():
    assert data.resolve_npairs(4096, 16, 0.03125) == 128
    assert data.resolve_npairs(4096, 16, 0.0) == 16
    assert data.resolve_npairs(16, 16, 0.03125) == 1


def test_asserts():
    import pytest
    g = torch.Generator().manual_seed(0)
    with pytest.raises(AssertionError):
        data.mqar_batch(1, 64, g, "cpu", n_pairs=64, n_queries=4, key_tokens=2)
    with pytest.raises(AssertionError):
        data.mqar_batch(1, 4096, g, "cpu", n_pairs=65, n_queries=1, key_tokens=1)


def test_passkey_and_copying_counts():
    g = torch.Generator().manual_seed(11)
    _, _, mask, pos = data.passkey_batch(2, 128, g, "cpu")
    assert int(mask.sum()) == 2 * data.KEY and pos is not None
    _, _, mask, pos = data.copying_batch(2, 128, g, "cpu")
    assert pos is None and int(mask.sum()) == 2 * (128 // 8)


def test_token_file(tmp_path):
    path = tmp_path / "tokens.bin"
    path.write_bytes(bytes(range(64)))
    ds = data.TokenDataset(path, "uint8")
    ids, target, mask, _ = ds.batch(2, 17, torch.Generator().manual_seed(0))
    torch.testing.assert_close(ids[:, 1:], target[:, :-1])
    assert tuple(mask.shape) == (2, 17)
