"""The batched pass's tcgen05 multi-column GEMM (`sp_mcol_gemm`) against a float64 reference of
the same arithmetic: W (fp16, or two fp16 halves) times x split into fp16 hi / lo halves, fp32
accumulation. Covers the whole-tile path (at least as many 128-row tiles as SMs) and the split-K
path (fewer tiles: partials summed in contributor order), partial row tiles, K that is not a multiple
of the 64-input k-block, up to four token tiles (T > 128), the three epilogues (store, residual add,
SwiGLU of interleaved gate / up rows) and two weight halves with a power-of-two alpha. Tolerance:
the fp32 accumulation bound 1e-5 x sum |w| |x| per output (the products themselves are exact)."""
import pytest
import torch

from seedplane_b200.config import PRESETS
from seedplane_b200.randinit import TEST_INIT, make_weights

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def engine():
    from seedplane_b200.engine import CudaQwen2
    cfg = PRESETS["tiny-hd64"]
    eng = CudaQwen2(cfg, make_weights(cfg, seed=0, dtype=torch.float16, **TEST_INIT), device="cuda:0")
    yield eng
    eng.close()


def ref(w, x, w_lo=None, alpha=1.0):
    """alpha * W . (hi + lo)^T in float64, with |W| . |x|^T for the error bound."""
    xs_hi = x.half()
    xs_lo = (x - xs_hi.float()).half()
    xd = xs_hi.double() + xs_lo.double()
    wd = w.double() + (w_lo.double() if w_lo is not None else 0.0)
    return alpha * (xd @ wd.T), abs(alpha) * (xd.abs() @ wd.abs().T)


def gen(N, K, T, seed, scale=0.05):
    g = torch.Generator().manual_seed(seed)
    w = (torch.randn((N, K), generator=g) * scale).half()
    x = torch.randn((T, K), generator=g)
    return w, x


@pytest.mark.parametrize("N,K,T", [(1152, 896, 16), (20000, 1536, 20), (896, 4864, 300), (1000, 200, 3),
                                   (151936, 256, 1), (2048, 1536, 512)])
def test_store_matches_float64(engine, N, K, T):
    w, x = gen(N, K, T, seed=N + K + T)
    got = engine.mcol_gemm(w.cuda(), x).cpu().double()
    want, bound = ref(w, x)
    err = (got - want).abs()
    assert torch.all(err <= 1e-5 * bound + 1e-30), float((err / (bound + 1e-30)).max())
    # deterministic: the same call again gives the same bits
    again = engine.mcol_gemm(w.cuda(), x).cpu().double()
    assert torch.equal(got, again)


def test_residual_add(engine):
    N, K, T = 896, 4864, 64
    w, x = gen(N, K, T, seed=3)
    y0 = torch.randn((T, N), generator=torch.Generator().manual_seed(4))
    y = y0.clone().cuda()
    engine.mcol_gemm(w.cuda(), x, mode="resid", y=y)
    want, bound = ref(w, x)
    err = (y.cpu().double() - (want + y0.double())).abs()
    assert torch.all(err <= 1e-5 * bound + 1e-6 * y0.abs().double() + 1e-30)


@pytest.mark.parametrize("N,K,T", [(1536, 256, 13), (17920, 1536, 40)])
def test_swiglu_interleaved(engine, N, K, T):
    w, x = gen(N, K, T, seed=5 + T)
    got = engine.mcol_gemm(w.cuda(), x, mode="swiglu").cpu().double()
    yd, bd = ref(w, x)
    g, u = yd[:, 0::2], yd[:, 1::2]
    silu = g / (1.0 + torch.exp(-g))
    want = silu * u
    # the GEMM's bound on gate and up carried through a = SiLU(g) u (|SiLU'| <= 1.1), plus the fp32
    # SwiGLU arithmetic and the fp16 hi + lo output (~2^-21 relative)
    eg, eu = 1e-5 * bd[:, 0::2], 1e-5 * bd[:, 1::2]
    tol = 1.1 * u.abs() * eg + silu.abs() * eu + 2e-6 * want.abs() + 1e-30
    assert torch.all((got - want).abs() <= tol), float(((got - want).abs() / tol).max())


def test_two_weight_halves_with_alpha(engine):
    N, K, T = 1024, 512, 40
    g = torch.Generator().manual_seed(9)
    wf = torch.randn((N, K), generator=g) * 40.0
    hi = wf.half()
    lo = (wf - hi.float()).half()
    x = torch.randn((T, K), generator=g)
    alpha = 2.0 ** -3
    got = engine.mcol_gemm(hi.cuda(), x, w_lo=lo.cuda(), alpha=alpha).cpu().double()
    want, bound = ref(hi, x, lo, alpha)
    assert torch.all((got - want).abs() <= 1e-5 * bound + 1e-30)


def test_no_device_error(engine):
    engine.status()
