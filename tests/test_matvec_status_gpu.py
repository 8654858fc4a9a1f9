"""The int8 tensor-core decode matvec's bounded waits: with every warp's first weight copy withheld (a copy that
never comes) and a short bound, the wait for it runs out; the launch then records SMOE_ETIMEOUT in the status word
the host reads (smoe_matvec_status), stops copying, lets its other copies in flight land, and the device stays
usable. Back to the default, the same call is exact again and leaves the status clear. No fault, no trap."""

import ctypes

import numpy as np
import pytest

from oracle import quants as Q

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def _status(lib, clear):
    v = ctypes.c_int(-1)
    assert lib.smoe_matvec_status(ctypes.byref(v), int(clear)) == 0
    return v.value


def test_a_wait_that_runs_out_is_a_status_the_host_reads(cuda):
    from strata_mlx_b200 import _lib
    from strata_mlx_b200 import blocks as B

    lib = _lib.lib()
    rng = np.random.default_rng(21)
    experts, rows, cols, pairs = 16, 1536, 4096, 8
    blocks = Q.random_blocks("IQ3_S", experts * rows * cols // 256, rng, normal=0.001).reshape(-1)
    lin = B.BlockSwitchLinear(torch.from_numpy(blocks).to(cuda), "IQ3_S", (experts, rows, cols))
    x = torch.from_numpy(rng.standard_normal((1, 1, 1, cols)).astype(np.float16)).to(cuda)  # a row shared by 8 pairs
    idx = torch.from_numpy(rng.choice(experts, size=(1, pairs), replace=False).astype(np.int32)).to(cuda)
    assert _status(lib, True) in (0, _lib.ETIMEOUT)  # (clear whatever an earlier test left)
    want = lin(x, idx)
    torch.cuda.synchronize()
    assert _status(lib, False) == 0
    try:
        assert lib.smoe_matvec_wait_test(2, 1) == 0
        for _ in range(3):
            lin(x, idx)
        assert _status(lib, True) == _lib.ETIMEOUT
    finally:
        assert lib.smoe_matvec_wait_test(-1, 0) == 0
    got = lin(x, idx)
    torch.cuda.synchronize()
    assert _status(lib, False) == 0
    assert torch.equal(got.view(torch.int16), want.view(torch.int16))
