"""The allocation-free GEMM entry point, called through its exported C symbol.

``dsv4_gemm_mx8_noalloc`` serves callers that may not allocate device memory
while they run (real-time loops that forbid cudaMalloc/cudaFree, which
synchronize the device; embedders with a fixed memory budget).  Its split-K scratch is a fixed array inside the library.  This test
checks it against the regular ``gemm`` binding (which takes a caller-allocated
workspace) on two calls in a row, since calls share and reuse the array, and
that oversized problems are refused without a launch.  The file sorts last so a
stop-at-first-failure run has already run every other test.
"""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

TOO_LARGE = -1


def _lib():
    from dsv4_flash_deployment_b200.ops import _ext

    _ext.load()  # the module is loaded once; ctypes reuses the same mapping
    lib = ctypes.CDLL(str(_ext.so_path()))
    fn = lib.dsv4_gemm_mx8_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p] * 5 + [ctypes.c_int] * 6 + [ctypes.c_void_p, ctypes.c_void_p]
    return fn


def _problem(m, n, k, seed):
    from dsv4_flash_deployment_b200.ops import gemm as G

    g = torch.Generator().manual_seed(seed)
    w = (torch.randn(m, k, generator=g) * 0.5).to(torch.float8_e4m3fn)
    s = torch.randint(118, 123, (m // 32, k // 32), generator=g, dtype=torch.int32).to(torch.uint8)
    x = torch.randn(n, k, generator=g).to(torch.bfloat16)
    mw = G.MxWeight.from_checkpoint(w, s, "cuda")
    xq, xsf = G.quantize(x.cuda())
    return mw, xq, xsf


def _call(fn, mw, xq, xsf, out, n, splits, err):
    stream = torch.cuda.current_stream().cuda_stream
    return fn(mw.q.data_ptr(), mw.sf.data_ptr(), xq.data_ptr(), xsf.data_ptr(), out.data_ptr(), mw.q.shape[0], n,
              mw.k, xq.shape[0], out.stride(0), splits, err.data_ptr(), stream)


def test_noalloc_matches_allocating_entry_point_twice():
    from dsv4_flash_deployment_b200.ops import gemm as G

    fn = _lib()
    m, n, k, splits = 512, 7, 2048, 4
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    for seed in (0, 1):  # two calls in a row share and reuse the scratch array
        mw, xq, xsf = _problem(m, n, k, seed)
        ref = torch.empty(n, m, dtype=torch.bfloat16, device="cuda")
        bn = G.pick_bn(n)
        tiles = (m // 128) * ((n + bn - 1) // bn)
        ws = torch.empty(tiles * splits * 128 * bn, dtype=torch.float32, device="cuda")
        cnt = torch.zeros(tiles, dtype=torch.int32, device="cuda")
        G.gemm_mx(xq, xsf, n, mw, ref, G.EPI_BF16, splits=splits, workspace=ws, counters=cnt)
        out = torch.full((n, m), float("nan"), dtype=torch.bfloat16, device="cuda")
        rc = _call(fn, mw, xq, xsf, out, n, splits, err)
        torch.cuda.synchronize()
        assert rc == 0, rc
        assert int(err.item()) == 0
        diff = (out.float() - ref.float()).abs()
        tol = 2e-2 * ref.float().abs() + 1e-2 * ref.float().abs().mean()
        assert bool((diff <= tol).all()), float(diff.max())


def test_noalloc_rejects_oversized_problem():
    fn = _lib()
    m, n, k = 4096, 256, 1024
    mw, xq, xsf = _problem(m, n, k, 2)
    out = torch.empty(n, m, dtype=torch.bfloat16, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    # 32 m-tiles x 1 n-tile x 8 splits x 128 x 256 floats = 8 Mi floats > 1 Mi
    assert _call(fn, mw, xq, xsf, out, n, 8, err) == TOO_LARGE
