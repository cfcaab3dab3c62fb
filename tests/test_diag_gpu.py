"""Device building blocks the hot kernels rely on, checked on the GPU through the C ABI:
the abort path of the bounded mbarrier wait (every wait in every kernel gives up
instead of hanging), and the FMA-pipe exponential of the attention softmax."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_bounded_wait_gives_up_records_its_site_and_the_kernel_returns():
    """A wait on a barrier that nothing completes, limited to 1 ms: the kernel returns
    (the stream synchronises), the fault word names the wait's site, the copy the kernel
    had in flight landed, its TMEM was released, and the context stays usable."""
    import torch
    from beacon_b200 import _lib, ops
    from beacon_b200.errors import LaunchError, check
    ops.device_status(0)  # start from clear fault words
    out = torch.zeros(3, dtype=torch.int32, device="cuda")
    check(_lib.lib().beacon_diag_wait_timeout(1_000_000, out.data_ptr(), torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    assert out.tolist() == [1, 1, 1]
    with pytest.raises(LaunchError):
        ops.device_status(0)
    assert "site 0x501" in _lib.last_error()
    assert ops.device_status(0) == (0, 0, 0)  # read and cleared
    # the context still runs kernels
    a = torch.ones(256, 256, dtype=torch.bfloat16, device="cuda")
    assert float(ops.matmul_fwd(a, a)[0, 0]) == 256.0
    assert _lib.lib().beacon_diag_wait_timeout(0, out.data_ptr(), None) == _lib.ERR_INVALID_LAUNCH_CONFIG


def test_fma_pipe_exp2_within_its_stated_bound():
    """exp2_poly2 against 2^x in float64.  On [-125.5, 8] (softmax arguments reach at most
    8 above the running maximum they are taken against) the relative error is below
    7.5e-5.  Below -125.5 the result nears the bottom of the float range (at -126 exactly
    the polynomial's value just under 1 lands in the subnormals) and arguments under -126
    are clamped: there the error stays below 2^-125 in absolute terms, far below anything
    a probability row that sums to at least 1 can register."""
    import torch
    from beacon_b200 import _lib
    from beacon_b200.errors import check
    x = np.concatenate([np.linspace(-125.5, 8.0, 1 << 20), np.arange(-125, 9, dtype=np.float64),
                        np.arange(-125, 8) + 0.5, np.linspace(-140.0, -125.5, 4096)]).astype(np.float32)
    if x.size % 2:
        x = np.append(x, np.float32(0.0))
    xin = torch.from_numpy(x).cuda()
    y = torch.empty_like(xin)
    check(_lib.lib().beacon_diag_exp2_poly(y.data_ptr(), xin.data_ptr(), x.size, None))
    torch.cuda.synchronize()
    got = y.cpu().numpy().astype(np.float64)
    ref = np.exp2(x.astype(np.float64))
    hi = x >= -125.5
    rel = np.abs(got[hi] - ref[hi]) / ref[hi]
    assert rel.max() < 7.5e-5, (rel.max(), x[hi][rel.argmax()])
    assert np.abs(got[~hi] - ref[~hi]).max() < 2.0 ** -125
