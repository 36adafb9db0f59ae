"""Lightning-indexer top-k kernels vs a plain PyTorch fp32 reference.

The reference scores every compressed entry j of token t as
``bf16(sum_h bf16(relu(bf16(q_h . k_j)) * w_h))`` (reference.py:605-702) and
takes the top-k.  The kernel sums heads in a fixed order and its dot products
accumulate in a different order than a PyTorch matmul, so scores may differ
by a bf16 ulp: the check is that the selected set is a top-k set of the
reference scores up to that tolerance, in ascending index order.
"""

import pytest
import torch

from dsv4_flash_deployment_b200.models.kv_format import ik4_decode, ik4_encode
from dsv4_flash_deployment_b200.ops import _ext
from dsv4_flash_deployment_b200.ops.gemm import ErrorWord

pytestmark = pytest.mark.gpu

HD = 128


def _keys(S, max_c):
    """Key cache as IK4 records on the device, and its exact decoded values (CPU)."""
    rec = ik4_encode(torch.randn(S, max_c, HD))
    return rec.cuda(), ik4_decode(rec, HD).bfloat16()


def _ref_scores(q, w, kc, slot, clen):
    out = []
    for t in range(q.shape[0]):
        k = kc[slot[t], :clen[t]].float()          # decoded key values
        raw = (q[t].float() @ k.T).bfloat16().float()                     # [H, clen]
        terms = (raw.clamp_min(0) * w[t, :, None]).bfloat16().float()
        out.append(terms.sum(0).bfloat16().float())
    return out


def _run(q, w, kc, slot, clen, topk, cand=None, cand_mode=0, cand_block=1, cand_topk=0):
    ext = _ext.load()
    T = q.shape[0]
    dev = q.device
    idx = torch.full((T, topk), -7, dtype=torch.int32, device=dev)
    cnt = torch.zeros(T, dtype=torch.int32, device=dev)
    keys = torch.empty(T, kc.shape[1], dtype=torch.int32, device=dev)
    ext.indexer_topk(q, w, kc, slot, clen, topk, idx, cnt, cand, cand_mode, cand_block, cand_topk, T,
                     ErrorWord.get(dev), None, None, None, None, 1, keys, None, None)
    torch.cuda.synchronize()
    ErrorWord.check(dev)
    return idx.cpu(), cnt.cpu()


def _check_topk(idx, cnt, scores, topk, allowed=None):
    for t, sc in enumerate(scores):
        n = sc.numel()
        if allowed is not None:
            sc = torch.where(allowed[t][:n], sc, torch.full_like(sc, float("-inf")))
        want = min(n, topk)
        assert int(cnt[t]) == want, (t, int(cnt[t]), want)
        sel = idx[t, :want]
        assert (idx[t, want:] == -1).all()
        assert (sel[1:] > sel[:-1]).all(), "indices must ascend"
        if n <= topk:
            assert torch.equal(sel, torch.arange(n, dtype=torch.int32))
            continue
        mask = torch.zeros(n, dtype=torch.bool)
        mask[sel.long()] = True
        lo = sc[mask].min()
        hi = sc[~mask].max()
        # one bf16 ulp of slack at the threshold
        ulp = torch.tensor(abs(float(lo)) if torch.isfinite(lo) else 0.0) * 2 ** -7
        assert float(lo) >= float(hi) - float(ulp) - 1e-6, (t, float(lo), float(hi))


@pytest.mark.parametrize("H", [8, 64])
@pytest.mark.parametrize("lens", [[5, 64, 65, 300], [2304, 1, 1000, 129]])
def test_indexer_topk_matches_reference(H, lens):
    torch.manual_seed(H + len(lens) + lens[0])
    dev = "cuda"
    topk = 64
    max_c = 2304
    S = 3
    T = len(lens)
    kc, kvals = _keys(S, max_c)
    q = torch.randn(T, H, HD).bfloat16().to(dev)
    w = (torch.randn(T, H) * 0.3).bfloat16().float().to(dev)
    slot = torch.tensor([i % S for i in range(T)], dtype=torch.int32, device=dev)
    clen = torch.tensor(lens, dtype=torch.int32, device=dev)
    idx, cnt = _run(q, w, kc, slot, clen, topk)
    ref = _ref_scores(q.cpu(), w.cpu(), kvals, slot.cpu(), lens)
    _check_topk(idx, cnt, ref, topk)


def test_indexer_candidate_blocks():
    """Level 1 builds a block mask from block maxima (newest block kept); level 2 selects inside it."""
    torch.manual_seed(3)
    dev = "cuda"
    topk, blk, ctop, max_c, H = 16, 16, 4, 512, 16
    lens = [500, 70, 33]
    T, S = len(lens), 2
    kc, kvals = _keys(S, max_c)
    q1 = torch.randn(T, H, HD).bfloat16().to(dev)
    q2 = torch.randn(T, H, HD).bfloat16().to(dev)
    w = (torch.rand(T, H) + 0.1).bfloat16().float().to(dev)
    slot = torch.tensor([0, 1, 0], dtype=torch.int32, device=dev)
    clen = torch.tensor(lens, dtype=torch.int32, device=dev)
    cand = torch.zeros(T, max_c // blk, dtype=torch.uint8, device=dev)
    _run(q1, w, kc, slot, clen, topk, cand, 1, blk, ctop)
    cand_cpu = cand.cpu().bool()
    ref1 = _ref_scores(q1.cpu(), w.cpu(), kvals, slot.cpu(), lens)
    allowed = []
    for t, sc in enumerate(ref1):
        n = sc.numel()
        nb = (n + blk - 1) // blk
        bmax = torch.stack([sc[b * blk:min(n, (b + 1) * blk)].max() for b in range(nb)])
        bmax[-1] = float("inf")
        got = cand_cpu[t, :nb]
        assert not cand_cpu[t, nb:].any()
        assert int(got.sum()) == min(nb, ctop)
        assert got[-1], "the newest block is always a candidate"
        if nb > ctop:
            lo, hi = bmax[got].min(), bmax[~got].max()
            assert float(lo) >= float(hi) - abs(float(hi)) * 2 ** -7 - 1e-6
        allowed.append(got.repeat_interleave(blk))
    idx, cnt = _run(q2, w, kc, slot, clen, topk, cand, 2, blk, ctop)
    ref2 = _ref_scores(q2.cpu(), w.cpu(), kvals, slot.cpu(), lens)
    for t in range(T):
        sel = idx[t, :int(cnt[t])].long()
        assert allowed[t][sel].all(), "level-2 picks stay inside candidate blocks"
    # entries outside the candidate blocks score -inf: the kept count may fall below topk
    for t, sc in enumerate(ref2):
        n = sc.numel()
        a = allowed[t][:n]
        want = min(n, topk)
        if n > topk:
            assert int(cnt[t]) == want
            chosen = torch.zeros(n, dtype=torch.bool)
            chosen[idx[t, :want].long()] = True
            in_a = sc.clone()
            in_a[~a] = float("-inf")
            if (chosen & a).any() and (a & ~chosen).any():
                lo = in_a[chosen & a].min()
                hi = in_a[a & ~chosen].max()
                assert float(lo) >= float(hi) - abs(float(hi)) * 2 ** -7 - 1e-6
