"""The tcgen05 W4A16 GEMM against a float64 product of the same dequantised
weights (the oracle's Q4 decode, quant_matmul.metal:39-47) and against the
CUDA-core GEMV it replaces at B > 1."""
import numpy as np
import pytest
import torch

from oracle import mirror as M
from tests._util import assert_close

pytestmark = pytest.mark.gpu


def _case(n, k, m, seed):
    rng = np.random.default_rng(seed)
    w = rng.normal(0, 0.02, (n, k)).astype(np.float32)
    packed, scales = M.q4_pack(w)
    x = rng.normal(0, 1, (m, k)).astype(np.float16)
    wd = M.q4_dequant(packed, scales, n, k).astype(np.float64)
    return packed, scales, x, wd


def _dev(packed, scales, x):
    return (torch.from_numpy(packed).cuda(), torch.from_numpy(scales.view(np.float16)).cuda(),
            torch.from_numpy(x).cuda())


@pytest.mark.parametrize("n,k,m", [(128, 64, 1), (256, 1536, 200), (2048, 1536, 128), (1536, 8960, 64),
                                   (384, 1536, 300), (65536, 512, 64), (65536, 512, 100), (65536, 512, 32)])
def test_w4a16_gemm_matches_dequantised_product(cuda, n, k, m):
    from llamamps_b200 import kernels as K
    packed, scales, x, wd = _case(n, k, m, seed=n + k + m)
    pk, sc, xd = _dev(packed, scales, x)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    y = K.w4a16_gemm(xd, pk, sc, n, k, error=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    ref = x.astype(np.float64) @ wd.T
    # fp16 weights (n - 8) * s carry up to 2^-11 relative rounding
    assert_close(y.cpu().numpy(), ref, abs_tol=2e-2, rel_tol=1e-2, what=f"gemm {m}x{n}x{k}")


@pytest.mark.parametrize("epi", ["none", "bias", "residual", "swiglu"])
def test_w4a16_gemm_persistent_equals_single_tiles(cuda, epi):
    """From 256 tokens the prefill GEMM is one persistent CTA per SM walking
    256 x 128 tiles (several per CTA here: 2085 tokens x 8960 rows = 630
    tiles), the accumulators alternating in TMEM.  Each output row sums the
    same K steps in the same order as the one-tile-per-CTA kernel (128 tokens
    per call), so the two agree bit for bit, for every epilogue and a ragged
    last tile."""
    from llamamps_b200 import kernels as K
    n, k, m = 8960, 1536, 2085
    packed, scales, x, wd = _case(n, k, m, seed=31)
    pk, sc, xd = _dev(packed, scales, x)
    rng = np.random.default_rng(32)
    kw = {}
    if epi == "bias":
        kw["bias"] = torch.from_numpy(rng.normal(0, 0.02, n).astype(np.float16)).cuda()
    if epi == "swiglu":
        kw["swiglu"] = True
    res = torch.from_numpy(rng.normal(0, 1, (m, n)).astype(np.float16)).cuda() if epi == "residual" else None
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    full = K.w4a16_gemm(xd, pk, sc, n, k, error=err, **kw, **({"residual": res} if res is not None else {}))
    mp = (m + 127) // 128 * 128
    xp = torch.zeros(mp, k, dtype=torch.float16, device="cuda")
    xp[:m] = xd
    rp = None
    if res is not None:
        rp = torch.zeros(mp, n, dtype=torch.float16, device="cuda")
        rp[:m] = res
    parts = []
    for r0 in range(0, mp, 128):
        extra = {"residual": rp[r0:r0 + 128].contiguous()} if rp is not None else {}
        parts.append(K.w4a16_gemm(xp[r0:r0 + 128].contiguous(), pk, sc, n, k, error=err, **kw, **extra))
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    ref = torch.cat(parts)[:m]
    assert full.shape == ref.shape
    assert torch.equal(full, ref), f"persistent vs single tiles differ ({epi})"


def test_w4a16_gemm_epilogues_and_gemv_agreement(cuda):
    from llamamps_b200 import kernels as K
    n, k, m = 256, 1536, 8
    packed, scales, x, wd = _case(n, k, m, seed=7)
    pk, sc, xd = _dev(packed, scales, x)
    rng = np.random.default_rng(8)
    bias = torch.from_numpy(rng.normal(0, 0.02, n).astype(np.float16)).cuda()
    res = torch.from_numpy(rng.normal(0, 1, (m, n)).astype(np.float16)).cuda()
    yb = K.w4a16_gemm(xd, pk, sc, n, k, bias=bias)
    yr = K.w4a16_gemm(xd, pk, sc, n, k, residual=res.clone())
    inplace = res.clone()
    K.w4a16_gemm(xd, pk, sc, n, k, residual=inplace, out=inplace)
    plain = x.astype(np.float64) @ wd.T
    assert_close(yb.cpu().numpy(), plain + bias.cpu().numpy(), what="bias epilogue")
    assert_close(yr.cpu().numpy(), res.cpu().numpy().astype(np.float64) + plain, what="residual epilogue")
    assert torch.equal(inplace, yr)
    # the CUDA-core GEMV (exact dequant) agrees within the fp16-weight rounding
    yg = K.gemv_q4(pk, sc, xd, n, k)
    assert_close(K.w4a16_gemm(xd, pk, sc, n, k).cpu().numpy(), yg.cpu().numpy(), what="gemm vs gemv")


@pytest.mark.parametrize("n,k,m", [(2048, 1536, 64), (1536, 8960, 64), (8960, 1536, 16), (256, 1536, 100),
                                   (128, 256, 3), (1536, 1536, 127)])
def test_w4a16_gemm_split_k(cuda, n, k, m):
    """Small-m calls split K over the CTAs of a cluster (fp32 partial tiles
    summed in distributed shared memory; trailing splits without K steps add
    zeros): residual epilogue against the float64 product, repeated calls
    give identical results."""
    from llamamps_b200 import kernels as K
    packed, scales, x, wd = _case(n, k, m, seed=3 * n + k + m)
    pk, sc, xd = _dev(packed, scales, x)
    rng = np.random.default_rng(5)
    res = torch.from_numpy(rng.normal(0, 1, (m, n)).astype(np.float16)).cuda()
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    ys = K.w4a16_gemm(xd, pk, sc, n, k, residual=res, error=err)
    y2 = K.w4a16_gemm(xd, pk, sc, n, k, residual=res, error=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    ref = res.cpu().numpy().astype(np.float64) + x.astype(np.float64) @ wd.T
    assert_close(ys.cpu().numpy(), ref, what=f"split-K gemm {m}x{n}x{k}")
    assert torch.equal(ys, y2)


def test_w4a16_gemm_rejects_unsupported_shapes(cuda):
    from llamamps_b200 import kernels as K
    x = torch.zeros(4, 64, dtype=torch.float16, device="cuda")
    pk = torch.zeros(100 * 32, dtype=torch.uint8, device="cuda")
    sc = torch.zeros(100 * 2, dtype=torch.float16, device="cuda")
    with pytest.raises(RuntimeError):
        K.w4a16_gemm(x, pk, sc, 100, 64)   # n not a multiple of 128
