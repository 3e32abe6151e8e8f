"""rt_column_order_device: the column cell order (headwater/src/sampler.rs:
655-668, cells by padding flag, column id, position) computed on the GPU must
equal the oracle's restatement bit for bit, as the host rt_column_order does."""
import ctypes

import numpy as np
import pytest

from oracle import rt_oracle as orc

pytestmark = pytest.mark.gpu


def device_order(col, pad):
    import torch
    from tributary_b200 import _lib
    b, s = col.shape
    col_d = torch.from_numpy(np.ascontiguousarray(col, dtype=np.int32)).cuda()
    pad_d = torch.from_numpy(np.ascontiguousarray(pad, dtype=np.uint8)).cuda()
    out = torch.full((b, s), -1, dtype=torch.int16, device="cuda")
    st = _lib.load().rt_column_order_device(col_d.data_ptr(), pad_d.data_ptr(), b, s, out.data_ptr(),
                                            ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    _lib.check(st, "rt_column_order_device")
    return out.cpu().numpy().view(np.uint16)


@pytest.mark.parametrize("gen", [
    (101, 4, 256, 3, 4, 8, 0.6, 0.05),
    (102, 3, 1000, 6, 4, 16, 0.7, 0.1),
    (103, 2, 4096, 24, 4, 16, 0.9, 0.05),
    (104, 2, 8192, 24, 4, 16, 0.9, 0.05),
    (105, 1, 16384, 6, 1, 3, 0.5, 0.3),
])
def test_device_column_order_matches_oracle(cuda_lib, gen):
    bt = orc.make_batch(*gen)
    np.testing.assert_array_equal(device_order(bt["column_ids"], bt["is_padding"]), bt["col_perm"])


def test_device_column_order_adversarial(cuda_lib):
    """Negative and repeated column ids, padding flags other than 0 / 1, a
    single cell, lengths that are not powers of two."""
    rng = np.random.default_rng(106)
    for s in (1, 3, 129, 777, 5000):
        col = rng.integers(-40, 40, (3, s)).astype(np.int32)
        col[1] = 7  # one column only: the order is padding, then position
        pad = rng.integers(0, 3, (3, s)).astype(np.uint8)
        want = np.stack([orc.compute_col_perm(col[b], pad[b]) for b in range(3)])
        np.testing.assert_array_equal(device_order(col, pad), want)


def test_device_column_order_length_limit(cuda_lib):
    import torch
    from tributary_b200 import _lib
    lib = _lib.load()
    col = torch.zeros(16385, dtype=torch.int32, device="cuda")
    pad = torch.zeros(16385, dtype=torch.uint8, device="cuda")
    out = torch.empty(16385, dtype=torch.int16, device="cuda")
    assert lib.rt_column_order_device(col.data_ptr(), pad.data_ptr(), 1, 16385, out.data_ptr(), None) == \
        _lib.RT_ERR_UNSUPPORTED
