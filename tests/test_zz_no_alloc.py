"""The allocation-free GEMM entry point, called through its exported C symbol.

``dsv4_gemm_mx8_noalloc`` (declared in ``csrc/dsv4_noalloc.h``) serves callers
that may not allocate device memory while they run: real-time loops that
forbid cudaMalloc/cudaFree, which can synchronize the device, and embedders
with a fixed memory budget.  Its split-K scratch is a fixed array inside the
library.  These tests check it against the regular ``gemm`` binding (which
takes a caller-allocated workspace) on two calls in a row, since calls share
and reuse the array, over split counts that use no scratch (1), divide the
k tiles, do not divide them, or leave the last splits without any k tile; and
that oversized problems and bad split counts are refused without touching the
output or the error word.  The return codes are read from the public header.
The file sorts last so a stop-at-first-failure run has already run every other
test.
"""

import ctypes
import re
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu

HEADER = Path(__file__).resolve().parent.parent / "dsv4_flash_deployment_b200" / "csrc" / "dsv4_noalloc.h"


def _codes():
    txt = HEADER.read_text()
    get = lambda name: int(re.search(rf"#define {name} \((-?\d+)\)", txt).group(1))
    return get("DSV4_NOALLOC_TOO_LARGE"), get("DSV4_NOALLOC_BAD_ARG")


def _lib():
    from dsv4_flash_deployment_b200.ops import _ext

    _ext.load()  # the module is loaded once; ctypes reuses the same mapping
    lib = ctypes.CDLL(str(_ext.so_path()))
    fn = lib.dsv4_gemm_mx8_noalloc
    fn.restype = ctypes.c_int
    # (a, a_sf, b, b_sf, out, m, n, k, b_rows, ldo, splits, err, stream), as in dsv4_noalloc.h
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


def _reference(mw, xq, xsf, n, m):
    """The allocating entry point without split-K: the GEMM every split count must match."""
    from dsv4_flash_deployment_b200.ops import gemm as G

    ref = torch.empty(n, m, dtype=torch.bfloat16, device="cuda")
    G.gemm_mx(xq, xsf, n, mw, ref, G.EPI_BF16, splits=1)
    return ref


@pytest.mark.parametrize("m,n,k,splits", [
    (512, 7, 2048, 4),     # 16 k tiles, even split
    (512, 7, 2048, 1),     # no split-K: the scratch is not used
    (256, 200, 2048, 3),   # n in 129..256 (256-token tile, two scale chunks); 6+6+4 k tiles
    (512, 7, 2048, 7),     # 3 k tiles per split: the 7th split has none and must add zeros
])
def test_noalloc_matches_allocating_entry_point_twice(m, n, k, splits):
    fn = _lib()
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    for seed in (0, 1):  # two calls in a row share and reuse the scratch array
        mw, xq, xsf = _problem(m, n, k, seed + 10 * splits)
        ref = _reference(mw, xq, xsf, n, m)
        out = torch.full((n, m), float("nan"), dtype=torch.bfloat16, device="cuda")
        rc = _call(fn, mw, xq, xsf, out, n, splits, err)
        torch.cuda.synchronize()
        assert rc == 0, rc
        assert int(err.item()) == 0
        diff = (out.float() - ref.float()).abs()
        tol = 2e-2 * ref.float().abs() + 1e-2 * ref.float().abs().mean()
        assert bool((diff <= tol).all()), float(diff.max())


def test_noalloc_rejects_oversized_problem_untouched():
    too_large, _ = _codes()
    fn = _lib()
    m, n, k = 4096, 256, 1024
    mw, xq, xsf = _problem(m, n, k, 2)
    out = torch.full((n, m), 3.0, dtype=torch.bfloat16, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    # 32 m-tiles x 1 n-tile x 8 splits x 128 x 256 floats = 8 Mi floats > 1 Mi
    assert _call(fn, mw, xq, xsf, out, n, 8, err) == too_large
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert bool((out == 3.0).all())


def test_noalloc_rejects_more_splits_than_k_tiles():
    _, bad_arg = _codes()
    fn = _lib()
    m, n, k = 256, 8, 512
    mw, xq, xsf = _problem(m, n, k, 3)
    out = torch.full((n, m), 3.0, dtype=torch.bfloat16, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    assert _call(fn, mw, xq, xsf, out, n, 5, err) == bad_arg   # 4 k tiles
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert bool((out == 3.0).all())
