"""Engram n-gram hashing (host, int64-exact).

States the hashing contract of the reference's ``engram_hash.py``
(``models/DeepSeekV4.1-Flash-v6e16/tpu-v7x/deepseek_v41/engram_hash.py:29-333``):

* a compressed token map: with a tokenizer, tokens whose decoded text
  normalizes to the same key share one compressed id (ids assigned in token-id
  order of first appearance, :func:`compressed_token_map`); without one,
  ``id % C``,
* per Engram layer, per n-gram order (2..max) and per head, a distinct prime
  modulus drawn in order layer -> order -> head, starting above
  ``engram_vocab_size - 1``; row offsets are the running sum of the primes,
* per-layer odd int64 multipliers from ``numpy.random.default_rng(10007*layer)``,
* for each token, the rolling XOR of ``token[t-k] * mult[k]`` (wrapping int64
  products), reduced mod each prime and shifted by its offset.

This module is the oracle for the native hasher in ``csrc/engram``.
"""

from __future__ import annotations

import re
import unicodedata
from dataclasses import dataclass
from pathlib import Path

import numpy as np

DEFAULT_COMPRESSED_VOCAB = 99092

_WS_RUN = re.compile(r"[ \t\r\n]+")
# characters with the Unicode White_Space property (what the strip removes;
# Python's own str.strip also removes U+001C..U+001F, which are not in it)
_WHITE_SPACE = "\t\n\x0b\x0c\r \x85\xa0\u1680" + "".join(map(chr, range(0x2000, 0x200B))) + \
    "\u2028\u2029\u202f\u205f\u3000"


def _fold_py(text: str) -> str:
    """The token-key normalization, restated with :mod:`unicodedata`.

    Compatibility composition (NFKC), then canonical decomposition (NFD) with
    the non-spacing marks dropped (accents), lowercase, every run of spaces,
    tabs and newlines collapsed to one space, and outer whitespace stripped --
    except that a text that is exactly one space stays one space.
    """
    s = unicodedata.normalize("NFD", unicodedata.normalize("NFKC", text))
    # marks dropped (non-spacing and enclosing); lowercase one character at a
    # time (no context-dependent final sigma)
    s = "".join(ch.lower() for ch in s if unicodedata.category(ch) not in ("Mn", "Me"))
    s = _WS_RUN.sub(" ", s)
    return s if s == " " else s.strip(_WHITE_SPACE)


def _fold_fn():
    """The normalizer that produced the trained tables' keys: the HuggingFace
    ``tokenizers`` normalizer sequence when that package is present (its Unicode
    tables and whitespace rules are the ones the checkpoint was built with),
    else the :mod:`unicodedata` restatement (which agrees with it except on
    characters whose Unicode properties differ between the two libraries'
    Unicode versions)."""
    try:
        from tokenizers import Regex, normalizers
    except ImportError:
        return _fold_py
    keep = "\ue000"   # private-use placeholder: a lone space survives the strip
    seq = normalizers.Sequence([
        normalizers.NFKC(), normalizers.NFD(), normalizers.StripAccents(), normalizers.Lowercase(),
        normalizers.Replace(Regex(r"[ \t\r\n]+"), " "), normalizers.Replace(Regex(r"^ $"), keep),
        normalizers.Strip(), normalizers.Replace(keep, " "),
    ])
    return seq.normalize_str


def _backend(tok):
    """(decode(id) -> str, token string of id, vocabulary size) of a tokenizer."""
    if isinstance(tok, (str, Path)):
        from tokenizers import Tokenizer
        p = Path(tok)
        if p.is_dir():
            p = p / "tokenizer.json"
        tok = Tokenizer.from_file(str(p))
        n = tok.get_vocab_size(with_added_tokens=True)
    elif hasattr(tok, "backend_tokenizer"):            # transformers fast tokenizer
        n = len(tok)
        tok = tok.backend_tokenizer
    else:
        n = tok.get_vocab_size(with_added_tokens=True) if hasattr(tok, "get_vocab_size") else len(tok)
    return (lambda i: tok.decode([i], skip_special_tokens=False)), tok.id_to_token, int(n)


def compressed_token_map(tokenizer=None, vocab_size: int = 129280,
                         compressed_vocab: int | None = None) -> tuple[np.ndarray, int]:
    """Token id -> compressed id table and the compressed vocabulary size.

    With a tokenizer (a ``tokenizer.json`` path or its directory, a
    ``tokenizers.Tokenizer``, a transformers fast tokenizer, or any object with
    ``decode``, ``id_to_token`` and a vocabulary size), each token's key is its
    decoded text after the normalization of :func:`_fold_fn`; a token that
    decodes to a partial UTF-8 sequence (U+FFFD in the text) keys on its raw
    token string instead, and one whose key normalizes to nothing keeps its
    text.  Keys get compressed ids in token-id order of first appearance.
    Behaviour of ``engram_hash.py:74-140``
    (``models/DeepSeekV4.1-Flash-v6e16/tpu-v7x/deepseek_v41/``).  Without a
    tokenizer: ``id % C`` with C = ``compressed_vocab`` (default 99092 for the
    129280-token vocabulary, else the vocabulary size).
    """
    if tokenizer is None:
        c = int(compressed_vocab or (DEFAULT_COMPRESSED_VOCAB if vocab_size == 129280 else vocab_size))
        return np.arange(vocab_size, dtype=np.int64) % c, c
    decode, raw, n = _backend(tokenizer)
    fold = _fold_fn()
    ids: dict[str, int] = {}
    table = np.empty(n, dtype=np.int64)
    for t in range(n):
        text = decode(t)
        if "\ufffd" in text:
            key = raw(t)
        else:
            key = fold(text) or text
        table[t] = ids.setdefault(key, len(ids))
    return table, len(ids)


def _is_prime(n: int) -> bool:
    """Deterministic Miller-Rabin for n < 3.3e24 (bases = first 12 primes)."""
    if n < 2:
        return False
    small = (2, 3, 5, 7, 11, 13, 17, 19, 23, 29, 31, 37)
    for p in small:
        if n % p == 0:
            return n == p
    d, r = n - 1, 0
    while d % 2 == 0:
        d //= 2
        r += 1
    for a in small:
        x = pow(a, d, n)
        if x in (1, n - 1):
            continue
        for _ in range(r - 1):
            x = x * x % n
            if x == n - 1:
                break
        else:
            return False
    return True


def next_unused_prime(start: int, used: set[int]) -> int:
    c = int(start) + 1
    while not _is_prime(c) or c in used:
        c += 1
    return c


@dataclass(frozen=True)
class EngramLayout:
    layer_ids: tuple[int, ...]
    max_ngram: int
    n_heads: int
    head_dim: int
    num_embeddings: tuple[int, ...]
    primes: np.ndarray    # [n_layers, max_ngram-1, n_heads] int64
    offsets: np.ndarray   # [n_layers, (max_ngram-1)*n_heads] int64

    @property
    def n_cols(self) -> int:
        return (self.max_ngram - 1) * self.n_heads

    @classmethod
    def from_config(cls, cfg) -> "EngramLayout | None":
        if not cfg.engram_layer_ids:
            return None
        used: set[int] = set()
        primes, offsets = [], []
        for _ in cfg.engram_layer_ids:
            per_order, flat = [], []
            for _ in range(cfg.engram_max_ngram_size - 1):
                cur = cfg.engram_vocab_size - 1
                row = []
                for _ in range(cfg.engram_n_heads):
                    cur = next_unused_prime(cur, used)
                    used.add(cur)
                    row.append(cur)
                per_order.append(row)
                flat.extend(row)
            primes.append(per_order)
            offsets.append(np.concatenate([[0], np.cumsum(flat[:-1])]).astype(np.int64))
        return cls(tuple(cfg.engram_layer_ids), cfg.engram_max_ngram_size, cfg.engram_n_heads,
                   cfg.engram_head_dim, tuple(cfg.engram_num_embeddings),
                   np.asarray(primes, dtype=np.int64), np.stack(offsets))


def hash_multipliers(layer_ids, max_ngram: int, compressed_vocab: int) -> np.ndarray:
    bound = max(1, (np.iinfo(np.int64).max // int(compressed_vocab)) // 2)
    rows = []
    for lid in layer_ids:
        g = np.random.default_rng(10007 * int(lid))
        rows.append(g.integers(0, bound, size=(max_ngram,), dtype=np.int64) * 2 + 1)
    return np.stack(rows) if rows else np.zeros((0, max_ngram), np.int64)


class EngramHasher:
    """Stateful per-sequence hasher: keeps the compressed token history."""

    DEAD = -1

    def __init__(self, cfg, compressed_vocab: int | None = None, token_map: np.ndarray | None = None):
        self.layout = EngramLayout.from_config(cfg)
        if self.layout is None:
            raise ValueError("config has no Engram layers")
        if token_map is None:
            token_map, c = compressed_token_map(None, cfg.vocab_size, compressed_vocab)
        else:
            c = int(token_map.max()) + 1
        self.compressed_vocab = c
        self.token_map = np.asarray(token_map, dtype=np.int64)
        self.pad = int(self.token_map[cfg.engram_pad_id])
        self.mult = hash_multipliers(self.layout.layer_ids, self.layout.max_ngram, c)

    def hash(self, history: np.ndarray, positions: np.ndarray) -> np.ndarray:
        """Row ids for tokens at ``positions`` of one sequence.

        history: compressed ids of the sequence so far (int64 [L]), already
        including the tokens being hashed.  Returns int64 [len(positions),
        n_engram_layers, n_cols].
        """
        lay = self.layout
        pos = np.asarray(positions, dtype=np.int64)
        toks = []
        blocked = np.zeros(pos.shape, dtype=bool)
        for shift in range(lay.max_ngram):
            src = history[np.maximum(pos - shift, 0)]
            blocked = blocked | (pos < shift) | (src == self.DEAD)
            toks.append(np.where(blocked, self.pad, src))
        t = np.stack(toks, -1)                                   # [P, n]
        with np.errstate(over="ignore"):
            prod = t[:, None, :] * self.mult[None, :, :]         # [P, nl, n] wrapping
        roll = prod[..., 0]
        out = []
        for i in range(1, lay.max_ngram):
            roll = np.bitwise_xor(roll, prod[..., i])
            out.append(roll[..., None] % lay.primes[None, :, i - 1, :])
        return np.concatenate(out, -1) + lay.offsets[None]

    def compress(self, token_ids) -> np.ndarray:
        return self.token_map[np.asarray(token_ids, dtype=np.int64)]
