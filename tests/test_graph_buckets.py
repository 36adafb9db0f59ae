"""Graph keys and bucketed step shapes (CPU).

A serving run changes its batch composition every step; the graph key must
depend only on what changes launch shapes, and padding to bucketed token /
sampled-row counts must keep the real rows first and only add work in the
scratch slot.
"""

import numpy as np

from dsv4_flash_deployment_b200.config import v4_flash_config
from dsv4_flash_deployment_b200.models.model import SeqChunk, StepMeta, token_bucket


def _cfg():
    return v4_flash_config(n_layers=4)


def test_token_bucket_sizes():
    assert [token_bucket(n, 4096) for n in (1, 2, 3, 5, 33, 64, 65, 127, 129, 1023)] == \
        [1, 2, 4, 8, 64, 64, 128, 128, 192, 1024]
    assert token_bucket(1000, 1010) == 1010      # capped at the buffer size
    assert token_bucket(2000, 1024) == 2000      # a count above the cap stays as it is
    assert token_bucket(0, 64) == 0


def test_key_ignores_chunk_lengths():
    cfg = _cfg()
    a = StepMeta(cfg, [SeqChunk(0, 100, [5]), SeqChunk(1, 0, list(range(40)))])
    b = StepMeta(cfg, [SeqChunk(0, 0, list(range(30))), SeqChunk(1, 200, list(range(11)))])
    assert a.T == b.T == 41
    assert a.key() == b.key()
    # a different chunk-count bucket changes the key (the compressor grid depends on it)
    c = StepMeta(cfg, [SeqChunk(i, 50, [i + 1]) for i in range(41)])
    assert c.key() != a.key()


def test_group_bound_covers_every_closed_group():
    cfg = _cfg()
    rng = np.random.default_rng(0)
    for _ in range(200):
        n = int(rng.integers(1, 12))
        chunks = [SeqChunk(i, int(rng.integers(0, 300)), [1] * int(rng.integers(1, 40))) for i in range(n)]
        m = StepMeta(cfg, chunks)
        for r, g in m.groups.items():
            assert len(g[0]) <= m.max_groups(r), (r, len(g[0]), m.max_groups(r))


def test_padded_step_keeps_real_rows_first():
    cfg = _cfg()
    m = StepMeta(cfg, [SeqChunk(0, 10, [7]), SeqChunk(1, 20, [8]), SeqChunk(2, 0, list(range(1, 38)))])
    p = m.padded(max_tokens=512, max_sample=512, pad_slot=9)
    assert m.T == 39 and p.T == 64
    assert p.n_out == 3 and len(p.sample_rows) == 4
    assert (p.sample_rows[:3] == m.sample_rows).all()
    assert (p.ids[:39] == m.ids).all() and (p.pos[:39] == m.pos).all() and (p.slot[:39] == m.slot).all()
    assert (p.slot[39:] == 9).all() and (p.pos[39:] == np.arange(25)).all()
    # two compositions of the same bucket replay one graph
    q = StepMeta(cfg, [SeqChunk(3, 5, list(range(1, 50))), SeqChunk(4, 7, [1]), SeqChunk(5, 9, [2])]).padded(512, 512, 9)
    assert q.key() == p.key()
    # never above the buffers
    big = StepMeta(cfg, [SeqChunk(0, 0, list(range(1, 500)))]).padded(max_tokens=500, max_sample=4, pad_slot=9)
    assert big.T == 500 and len(big.sample_rows) == 1


def test_padded_meta_extends_every_array_of_the_step():
    """The padded step keeps every real token's and sampled row's values and
    appends the padding chunk (positions 0.. of the pad slot, not sampled)."""
    import numpy as np

    from dsv4_flash_deployment_b200.config import toy_v4_config
    from dsv4_flash_deployment_b200.models.model import SeqChunk, StepMeta

    cfg = toy_v4_config()
    rng = np.random.default_rng(3)
    for trial in range(20):
        chunks = []
        for i in range(int(rng.integers(1, 9))):
            n = int(rng.integers(1, 12))
            chunks.append(SeqChunk(i, int(rng.integers(0, 40)), rng.integers(0, 1000, n).tolist(), bool(rng.random() < .8),
                                   sample_all=bool(rng.random() < .2), temperature=float(rng.choice([0.0, 0.7])),
                                   top_k=int(rng.choice([0, 5])), seed=None if rng.random() < .5 else int(trial)))
        m = StepMeta(cfg, chunks)
        p = m.padded(64, 64, 9)
        T, S = m.T, len(m.sample_rows)
        for name in ("ids", "pos", "slot", "chunk_start", "step_row0", "last_pos"):
            assert np.array_equal(getattr(p, name)[:T], getattr(m, name)), name
        assert p.T >= T and (p.ids[T:] == 0).all() and (p.slot[T:] == 9).all()
        assert np.array_equal(p.pos[T:], np.arange(p.T - T))
        for name in ("sample_rows", "temps", "topk", "topp", "seedkey", "has_seed"):
            assert np.array_equal(getattr(p, name)[:S], getattr(m, name)), name
        assert p.n_out == S and p.lp_want[:S] == m.lp_want
        assert (p.sampling, p.filtering, p.seeded) == (m.sampling, m.filtering, m.seeded)
        # the same step built directly from its chunks
        q = StepMeta(cfg, p.chunks)
        for name in ("ids", "pos", "slot", "last_pos"):
            assert np.array_equal(getattr(q, name), getattr(p, name)), name
