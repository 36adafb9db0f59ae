"""Debug-bounds build (``DSV4_DEBUG_BOUNDS=1``): the cache gathers check their
indices and report a bad one in the device error word instead of reading
outside the cache.  Runs in a child process (the extension variant is chosen
when the library loads).  The bad index used here, entry ``max_c`` of slot 0
of a contiguous 3-slot cache, would land on row 0 of slot 1, inside the
allocation, even in a build without the check."""

import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu


def _child() -> None:
    import torch

    from dsv4_flash_deployment_b200.engine.builder import build_model
    from dsv4_flash_deployment_b200.io.checkpoint_spec import make_random_weights
    from dsv4_flash_deployment_b200.models.model import SeqChunk, StepMeta
    from dsv4_flash_deployment_b200.ops import _ext
    from dsv4_flash_deployment_b200.ops.gemm import ErrorWord
    from test_model_gpu import small_v4

    ext = _ext.load()
    assert ext.debug_bounds, "debug-bounds extension not loaded"
    cfg = small_v4()
    m = build_model(cfg, "cuda", max_tokens=64, n_slots=2, max_seq_len=64, weights=make_random_weights(cfg, seed=3))
    seq = [(7 * i) % 1000 + 16 for i in range(40)]
    for meta in (StepMeta(cfg, [SeqChunk(0, 0, seq, True)]), StepMeta(cfg, [SeqChunk(0, 40, [21], True)])):
        m.upload(meta)
        m.forward(meta)
        torch.cuda.synchronize()
        ErrorWord.check("cuda")            # valid indices: nothing reported
    lid = 1                                 # ratio-4 kv source
    comp = m.comp[lid]
    max_c = comp.shape[1]
    idx = torch.zeros(1, cfg.index_topk, dtype=torch.int32, device="cuda")
    idx[0, 0] = max_c                       # one past the slot's last entry
    cnt = torch.tensor([2], dtype=torch.int32, device="cuda")
    cos, sin = m.rope["yarn"]
    ext.attention(m.q, cos, sin, None, cfg.q_head_norm, cfg.rms_norm_eps, m.kv_step, m.ring[lid], comp, m.m_slot,
                  m.m_pos, m.m_cstart, m.m_row0, idx, cnt, m.layers[lid].sink, cfg.head_dim ** -0.5, m.o, None, 1, 1,
                  None, 0, None)
    torch.cuda.synchronize()
    try:
        ErrorWord.check("cuda")
        raise AssertionError("bad cache index not reported")
    except RuntimeError as e:
        msg = str(e)
    assert "code=3" in msg and "kernel=6" in msg and "detail=1" in msg, msg
    # the context is still usable
    meta = StepMeta(cfg, [SeqChunk(0, 41, [22], True)])
    m.upload(meta)
    m.forward(meta)
    torch.cuda.synchronize()
    ErrorWord.check("cuda")
    print("DEBUG_BOUNDS_OK", flush=True)


def test_debug_bounds_build_reports_a_bad_cache_index():
    from dsv4_flash_deployment_b200.ops import _ext

    assert _ext.so_path(dbg=True).exists(), "debug-bounds extension not built (__graft_entry__.build())"
    env = dict(os.environ, DSV4_DEBUG_BOUNDS="1")
    r = subprocess.run([sys.executable, __file__], capture_output=True, text=True, env=env, timeout=600,
                       cwd=os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    assert r.returncode == 0 and "DEBUG_BOUNDS_OK" in r.stdout, r.stdout[-3000:] + r.stderr[-3000:]


if __name__ == "__main__":
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    _child()
