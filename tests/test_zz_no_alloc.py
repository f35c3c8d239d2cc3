"""`sp_argmax_noalloc` (fixed device scratch, no allocation per call) against `sp_argmax`.

Two calls in a row on the same inputs must both equal the engine entry point's result: the second
call checks that the first left the fixed scratch usable (the row counters are cleared before each
launch and reset by the kernel). Oversize requests are rejected before anything is launched."""
import numpy as np
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


def cases(seed=1):
    g = np.random.default_rng(seed)
    out = []
    for rows, cols, ld in ((1, 151936, 151936), (128, 1000, 1000), (7, 8193, 8195), (3, 5, 5), (128, 20000, 20004)):
        x = g.standard_normal((rows, ld)).astype(np.float32)
        for r in range(rows):
            a, b = sorted(int(v) for v in g.integers(0, cols, 2))
            x[r, a] = x[r, b] = 7.5                  # tie: the lower index wins
            x[r, cols:] = 50.0                       # beyond `cols`: ignored
        out.append((x, cols))
    return out


def test_noalloc_twice_equals_engine_argmax(engine):
    from seedplane_b200.engine import argmax_noalloc
    for x, cols in cases():
        dev = torch.from_numpy(x).to(engine.device)[:, :cols]
        want = engine.argmax(dev)
        first = argmax_noalloc(dev)
        second = argmax_noalloc(dev)
        torch.cuda.synchronize()
        assert torch.equal(first, want) and torch.equal(second, want)
        assert (want.cpu().numpy() == np.argmax(x[:, :cols], axis=1)).all()


def test_noalloc_rejects_oversize_without_launching(engine):
    from seedplane_b200.engine import argmax_noalloc
    x = torch.zeros((129, 16), dtype=torch.float32, device=engine.device)
    with pytest.raises(ValueError, match="at most 128 rows"):
        argmax_noalloc(x)
    # still usable afterwards
    x[:, 3] = 1.0
    assert (argmax_noalloc(x[:128]) == 3).all()


def test_noalloc_rejects_host_buffers_and_keeps_the_current_device(engine):
    """Host memory is refused before anything is launched, and the calling thread's current device
    is the same after a call as before it."""
    import ctypes as C
    from seedplane_b200 import _native as N
    before = torch.cuda.current_device()
    host = torch.zeros((2, 16), dtype=torch.float32)
    out = torch.zeros(2, dtype=torch.int32, device=engine.device)
    rc = N.load().sp_argmax_noalloc(engine.device.index or 0, C.c_void_p(host.data_ptr()), 2, 16, 16,
                                    C.c_void_p(out.data_ptr()), None)
    assert rc != 0 and "device memory" in N.load().sp_last_error().decode()
    assert torch.cuda.current_device() == before
