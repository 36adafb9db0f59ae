"""Small device kernels vs plain PyTorch references: row argmax (single- and multi-CTA
rows); the decode-step router (gate GEMV + top-k in one launch)."""

import pytest
import torch

from dsv4_flash_deployment_b200.ops import _ext

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("T", [1, 3, 40, 200])
@pytest.mark.parametrize("V", [1000, 129280, 129283])
def test_argmax_rows_matches_torch(T, V):
    ext = _ext.load()
    torch.manual_seed(T * 7 + V)
    ld = (V + 127) // 128 * 128 + (1 if V % 2 else 0)   # odd V: unaligned rows take the scalar path
    logits = torch.randn(T, ld, device="cuda")
    # ties: the first index wins
    logits[:, 5] = 9.0
    logits[:, V - 3] = 9.0
    logits[T // 2, :] = 0.0
    logits[T // 2, V - 1] = 1.0
    scratch = torch.zeros(2 * max(T, 296) + 256, dtype=torch.int32, device="cuda")
    for use_scratch in (False, True):
        out = torch.full((T,), -1, dtype=torch.int32, device="cuda")
        for _ in range(3):   # counters must come back to zero between calls
            ext.argmax_rows(logits, T, V, out, scratch if use_scratch else None, None, 0)
        want = torch.argmax(logits[:, :V], dim=1).int()
        torch.cuda.synchronize()
        assert torch.equal(out, want)
    assert int(scratch[-256:].abs().sum()) == 0


@pytest.mark.parametrize("T", [1, 4])
@pytest.mark.parametrize("E,D,k,score_func", [(256, 4096, 8, 0), (384, 5120, 6, 1)])
def test_router_small_matches_reference(T, E, D, k, score_func):
    """Logits = u . gate^T (fp32 accumulation of bf16 products), then the same top-k
    as router_topk on those logits: picks and weights equal the reference routing of
    the kernel's own logits, and the logits match an fp32 matmul to rounding."""
    ext = _ext.load()
    g = torch.Generator(device="cuda").manual_seed(T + E)
    u = torch.randn(T, D, device="cuda", generator=g).to(torch.bfloat16)
    w = (torch.randn(E, D, device="cuda", generator=g) * D ** -0.5).to(torch.bfloat16)
    bias = torch.randn(E, device="cuda", generator=g) * 0.1
    logits = torch.zeros(T, E, device="cuda")
    ids = torch.zeros(T, k, dtype=torch.int32, device="cuda")
    wts = torch.zeros(T, k, device="cuda")
    counter = torch.zeros(1, dtype=torch.int32, device="cuda")
    for _ in range(3):   # the counter must come back to zero
        ext.router_small(u, w, T, logits, bias, k, score_func, 1.5, ids, wts, counter)
    torch.cuda.synchronize()
    assert int(counter) == 0
    want = u.float() @ w.float().t()
    assert float((logits - want).abs().max()) < 1e-3 * float(want.abs().max())
    ids2 = torch.zeros_like(ids)
    wts2 = torch.zeros_like(wts)
    ext.router_topk(logits, T, bias, k, score_func, 1.5, ids2, wts2)
    torch.cuda.synchronize()
    assert torch.equal(ids, ids2) and torch.equal(wts, wts2)


def _probe(ext, graph: bool):
    ctas = 64
    stamps = torch.zeros(1 + 2 * ctas, dtype=torch.int64, device="cuda")
    if graph:
        g = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            with torch.cuda.graph(g, stream=s):
                ext.pdl_probe(stamps, ctas, 200_000)
        torch.cuda.current_stream().wait_stream(s)
        g.replay()
    else:
        # the engine runs on its own stream (the legacy default stream serializes)
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            ext.pdl_probe(stamps, ctas, 200_000)
    torch.cuda.synchronize()
    st = stamps.cpu()
    end_first = int(st[0])
    entries = st[1::2][:ctas]
    exits = st[2::2][:ctas]
    return end_first, entries, exits


@pytest.mark.parametrize("graph", [False, True])
def test_programmatic_launch_overlaps_and_orders(graph):
    """Every kernel starts with griddepcontrol.launch_dependents + wait: nothing
    after the wait starts before the previous kernel has finished (eager and graph
    replay), and in a graph replay (how the engine runs its steps) the next
    kernel's CTAs are already scheduled while the previous one still runs.
    Eager launches on this driver showed no early start, so that half is only
    asserted for graphs."""
    import os

    ext = _ext.load()
    end_first, entries, exits = _probe(ext, graph)
    assert int(exits.min()) >= end_first, "a dependent passed griddepcontrol.wait before its predecessor ended"
    if graph and os.environ.get("DSV4_PDL", "1") != "0":
        assert int(entries.min()) < end_first, "dependent grid was not launched early"
