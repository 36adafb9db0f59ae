"""Sampling rules of the head: temperature (Gumbel-max), top-k / top-p nucleus
filtering and log-probabilities.

Every function works on a ``[S, V]`` fp32 logits tensor on any device, so the
device model (``DSV4Model`` in model.py, inside its captured CUDA graph) and the
CPU oracle step (oracle_step.py) apply the same rule and the CPU tests check
the one the GPU runs.  They are torch operations on the sampled rows only (a
few hundred rows at most); the head GEMM and the argmax stay in this library's
kernels.

The reference's own server decodes greedily (``tpu-v7x/deepseek_v41/server.py:
44-150``); the vLLM-served recipes inherit vLLM's sampler, whose order this
follows: log-probabilities come from the raw logits (vLLM's default
``logprobs_mode``), top-k is applied before top-p, and top-p keeps the smallest
prefix of the temperature-scaled, top-k-truncated distribution whose mass
reaches ``p`` (at least one token).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

LOGPROB_TOP_N = 20   # most alternatives a request may ask for (the OpenAI API's top_logprobs limit)


@dataclass(frozen=True)
class SamplingParams:
    """Per-request decoding rule.  ``temperature`` 0 is greedy (top-k / top-p then
    change nothing); ``top_k`` 0 and ``top_p`` 1.0 are off; ``logprobs`` None asks
    for none, n >= 0 for the sampled token's log-probability plus the n most
    likely alternatives; ``seed`` makes the request's samples a function of
    (seed, position) only (:func:`seeded_gumbel`), whatever it is batched with."""

    temperature: float = 0.0
    top_k: int = 0
    top_p: float = 1.0
    logprobs: int | None = None
    seed: int | None = None

    def __post_init__(self):
        if self.temperature < 0:
            raise ValueError("temperature must be >= 0")
        if self.top_k < 0:
            raise ValueError("top_k must be >= 0 (0: off)")
        if not 0.0 < self.top_p <= 1.0:
            raise ValueError("top_p must be in (0, 1]")
        if self.logprobs is not None and not 0 <= self.logprobs <= LOGPROB_TOP_N:
            raise ValueError(f"logprobs must be between 0 and {LOGPROB_TOP_N}")

    @property
    def filters(self) -> bool:
        """True when top-k / top-p can change the sample (only under temperature > 0)."""
        return self.temperature > 0 and (self.top_k > 0 or self.top_p < 1.0)

    @property
    def wants_logprobs(self) -> bool:
        return self.logprobs is not None


def gumbel_(logits: torch.Tensor, temps: torch.Tensor, noise: torch.Tensor,
            seeded: tuple[torch.Tensor, torch.Tensor] | None = None, v0: int = 0) -> None:
    """In place: ``logits += temps * g`` with g ~ Gumbel(0, 1) drawn into ``noise``
    (same shape).  The argmax of the result is a sample of softmax(logits / T);
    rows at T = 0 are unchanged (greedy).  ``seeded`` = (row keys int64 [S], row
    has a seed bool [S]): those rows take :func:`seeded_gumbel` noise for
    vocabulary columns ``v0 ..`` instead of the device generator's."""
    noise.uniform_(1e-20, 1.0 - 1e-7)
    noise.log_().neg_().log_().neg_()
    if seeded is not None:
        keys, has = seeded
        noise.copy_(torch.where(has[:, None], seeded_gumbel(keys, noise.shape[1], v0), noise))
    logits.addcmul_(temps[:, None], noise)


# SplitMix64 (G. Steele, D. Lea, C. Flood, "Fast splittable pseudorandom number
# generators", OOPSLA 2014): the golden-ratio increment and the two multipliers
# of its output mix, as signed 64-bit values (torch has no unsigned int64).
def _s64(x: int) -> int:
    x &= (1 << 64) - 1
    return x - (1 << 64) if x >> 63 else x


_SM_GAMMA = _s64(0x9E3779B97F4A7C15)
_SM_M1 = _s64(0xBF58476D1CE4E5B9)
_SM_M2 = _s64(0x94D049BB133111EB)


def _srl(x: torch.Tensor, k: int) -> torch.Tensor:
    """Logical right shift of int64 values (torch's >> is arithmetic)."""
    return (x >> k) & ((1 << (64 - k)) - 1)


def _mix(z: torch.Tensor) -> torch.Tensor:
    z = (z ^ _srl(z, 30)) * _SM_M1
    z = (z ^ _srl(z, 27)) * _SM_M2
    return z ^ _srl(z, 31)


def splitmix64(x: int) -> int:
    """The SplitMix64 output for state ``x`` (host integers, exact mod 2^64)."""
    m = (1 << 64) - 1
    z = (x + 0x9E3779B97F4A7C15) & m
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & m
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & m
    return z ^ (z >> 31)


def seed_key(seed: int, position: int) -> int:
    """Per (request seed, token position) key of the seeded noise, as a signed int64."""
    return _s64(splitmix64(splitmix64(seed & ((1 << 64) - 1)) ^ (position & ((1 << 64) - 1))))


def seeded_gumbel(keys: torch.Tensor, n: int, v0: int = 0) -> torch.Tensor:
    """Gumbel(0, 1) noise [S, n] for vocabulary columns v0 .. v0 + n - 1: entry
    (s, v) is a function of keys[s] and v only (SplitMix64 of key + v * gamma, top
    24 bits as a uniform in (0, 1)), the same on every device and under any
    vocabulary split."""
    v = torch.arange(v0, v0 + n, device=keys.device, dtype=torch.int64)
    z = _mix(keys[:, None] + v[None, :] * _SM_GAMMA)
    u = (_srl(z, 40).to(torch.float32) + 0.5) * (1.0 / (1 << 24))
    return -torch.log(-torch.log(u))


def top_k_top_p_mask_(logits: torch.Tensor, temps: torch.Tensor, top_k: torch.Tensor, top_p: torch.Tensor) -> None:
    """In place: every entry outside the row's top-k set or top-p nucleus becomes
    -inf.  ``top_k`` (int, 0 = off) and ``top_p`` (float, >= 1 = off) are per row;
    the nucleus is taken over softmax(logits / T) after the top-k cut (T = 1 for
    greedy rows, which no cut can change).  Entries tied with a row's threshold
    stay."""
    S, V = logits.shape
    if S == 0:
        return
    srt = torch.sort(logits, dim=-1, descending=True).values
    k = torch.where(top_k > 0, top_k.clamp(max=V), torch.full_like(top_k, V)).long()
    thr_k = srt.gather(1, (k - 1)[:, None])
    rank = torch.arange(V, device=logits.device)
    t = torch.where(temps > 0, temps, torch.ones_like(temps))
    z = (srt / t[:, None]).masked_fill(rank[None, :] >= k[:, None], float("-inf"))
    p = torch.softmax(z, dim=-1)
    before = p.cumsum(-1) - p                    # mass of the strictly more likely entries
    n_keep = (before < top_p[:, None]).sum(-1).clamp(min=1)
    thr_p = srt.gather(1, (n_keep - 1)[:, None])
    thr_p = torch.where(top_p[:, None] >= 1.0, torch.full_like(thr_p, float("-inf")), thr_p)
    logits.masked_fill_(logits < torch.maximum(thr_k, thr_p), float("-inf"))


def logprob_top(logits: torch.Tensor, n: int) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """(logsumexp [S], top-n log-probabilities [S, n], their token ids [S, n]) of
    raw logits."""
    lse = torch.logsumexp(logits, dim=-1)
    vals, ids = torch.topk(logits, n, dim=-1)
    return lse, vals - lse[:, None], ids


def chosen_logprob(raw: torch.Tensor, ids: torch.Tensor, lse: torch.Tensor) -> torch.Tensor:
    """Log-probability [S] of token ``ids[s]`` under raw logits ``raw[s]``."""
    return raw.gather(1, ids.long()[:, None])[:, 0] - lse


def logprob_entries(chosen: list[float], vals: list[list[float]], ids: list[list[int]],
                    want: list[int | None]) -> list[dict | None]:
    """Host records per sampled row: ``{"logprob": float, "top": [(id, lp), ...]}``
    with the row's requested number of alternatives, or None where a row asked
    for none."""
    out = []
    for i, n in enumerate(want):
        if n is None:
            out.append(None)
            continue
        out.append({"logprob": float(chosen[i]), "top": [(int(t), float(v)) for t, v in zip(ids[i][:n], vals[i][:n])]})
    return out
