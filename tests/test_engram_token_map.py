"""Engram compressed token map built from a tokenizer (CPU).

Tokens whose decoded text normalizes to one key (NFKC, accents stripped,
lowercase, whitespace runs collapsed, outer whitespace stripped, a lone space
kept) share a compressed id; ids follow token-id order of first appearance; a
token decoding to a partial UTF-8 sequence keys on its raw token string.  The
expected tables below are worked out by hand from those rules.
"""

import json

import numpy as np
import pytest

from dsv4_flash_deployment_b200.ref import engram as E

VOCAB = ["<unk>", "Hello", "hello", "HELLO", "Héllo", " ", "\t", "  ", "ﬁne", "fine", "Straße",
         "x\ny", "x y", "café", "cafe", "  Word　"]
#         0        1        2        3        4             5    6     7     8 (fi ligature) 9   10
#         11      12      13              14      15 (nbsp / ideographic space around it)
EXPECTED = [0, 1, 1, 1, 1, 2, 2, 2, 3, 3, 4, 5, 5, 6, 6, 7]


def _tokenizer_json(path):
    tokenizers = pytest.importorskip("tokenizers")
    from tokenizers import Tokenizer, models

    tok = Tokenizer(models.WordLevel({t: i for i, t in enumerate(VOCAB)}, unk_token="<unk>"))
    tok.save(str(path))
    # the file is plain JSON: the fixture is what a checkpoint ships
    json.loads(path.read_text())
    return path


def test_token_map_from_tokenizer_json(tmp_path):
    p = _tokenizer_json(tmp_path / "tokenizer.json")
    table, c = E.compressed_token_map(str(p))
    assert c == 8
    assert table.tolist() == EXPECTED
    # directory form and the Tokenizer object give the same table
    t2, c2 = E.compressed_token_map(str(tmp_path))
    assert (t2 == table).all() and c2 == c


def test_python_restatement_agrees_with_tokenizers_normalizer():
    pytest.importorskip("tokenizers")
    fold = E._fold_fn()
    for text in VOCAB + ["AΣ", "İstanbul", "Ⅻ", "  \t\n x  ", "\x1c", "", "Ångström"]:
        assert E._fold_py(text) == fold(text), repr(text)


class _ByteTokens:
    """Tokenizer double: two ids decode to a lone continuation byte (U+FFFD)."""

    texts = ["a", "�", "A", "�", ""]
    raw = ["a", "<0xE2>", "A", "<0xE3>", "<pad>"]

    def decode(self, ids, skip_special_tokens=False):
        assert not skip_special_tokens
        return self.texts[ids[0]]

    def id_to_token(self, i):
        return self.raw[i]

    def __len__(self):
        return len(self.texts)


def test_partial_utf8_tokens_key_on_raw_string():
    table, c = E.compressed_token_map(_ByteTokens())
    # "a" and "A" share a key; the two partial bytes differ by raw string; "" keeps its text
    assert table.tolist() == [0, 1, 0, 2, 3]
    assert c == 4


def test_no_tokenizer_is_modulo():
    table, c = E.compressed_token_map(None, vocab_size=129280)
    assert c == E.DEFAULT_COMPRESSED_VOCAB
    assert table[99092] == 0 and table[5] == 5
    table, c = E.compressed_token_map(None, vocab_size=1000, compressed_vocab=7)
    assert c == 7 and (table == np.arange(1000) % 7).all()


def test_hasher_uses_the_tokenizer_map():
    from dsv4_flash_deployment_b200.config import v41_tiny_config

    cfg = v41_tiny_config()
    assert cfg.engram_layer_ids
    table = np.arange(cfg.vocab_size, dtype=np.int64) // 2     # pairs of tokens share an id
    h = E.EngramHasher(cfg, token_map=table)
    assert h.compressed_vocab == int(table.max()) + 1
    assert (h.compress([0, 1, 2, 3]) == [0, 0, 1, 1]).all()

