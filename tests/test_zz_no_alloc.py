"""efg_host_matvec_static: the host-pointer matvec staged through the library's static
device area. Named to be collected last; it also passes on its own."""
from __future__ import annotations

import numpy as np
import pytest

import edgeforge_b200 as efg
from edgeforge_b200 import QType

pytestmark = pytest.mark.gpu


def _case(qt, rows, cols, seed):
    rng = np.random.default_rng(seed)
    W = efg.host_quantize_row(qt, (0.02 * rng.standard_normal(rows * cols)).astype(np.float32))
    x = rng.standard_normal(cols).astype(np.float32)
    return W, x


@pytest.mark.parametrize("qt,rows,cols", [(QType.Q4_0, 5632, 2048), (QType.Q8_0, 1000, 2048), (QType.Q4_0, 37, 96)])
def test_static_matches_host_matvec_twice(qt, rows, cols, oracle):
    """Two calls in a row with different inputs: each result equals efg_host_matvec's bit
    for bit and is within the reference's 1e-5 of sum|w x| of the exact dot."""
    import torch

    from conftest import rel_dot_errors

    for call, seed in enumerate((1, 2)):  # two calls in a row, different inputs
        W, x = _case(qt, rows, cols, seed)
        want = efg.host_matvec(qt, W, x, rows)
        if call == 1:
            free0 = torch.cuda.mem_get_info(0)[0]
        got = efg.host_matvec_static(qt, W, x, rows)
        np.testing.assert_array_equal(got, want)
        if call == 1:
            assert torch.cuda.mem_get_info(0)[0] == free0  # nothing allocated by the call
        err = rel_dot_errors(oracle, qt, W.reshape(rows, -1), x, rows, got)
        assert err.max() <= 1e-5, err.max()
    assert efg.device_error() == 0


def test_static_rejects_oversize_and_bad_args():
    W, x = _case(QType.Q8_0, 32, 2048, 3)
    with pytest.raises(efg.EdgeForgeError, match="static area holds"):
        efg.host_matvec_static(QType.Q8_0, np.zeros(32000 * 2176, np.uint8), x, 32000)
    with pytest.raises(efg.EdgeForgeError, match="divisible by 32"):
        efg.host_matvec_static(QType.Q4_0, W, x[:30], 1)
    with pytest.raises(efg.EdgeForgeError, match="not a packed type"):
        efg.host_matvec_static(QType.F32, W, x, 32)
    # the area is still usable after a rejected call
    np.testing.assert_array_equal(efg.host_matvec_static(QType.Q8_0, W, x, 32), efg.host_matvec(QType.Q8_0, W, x, 32))
