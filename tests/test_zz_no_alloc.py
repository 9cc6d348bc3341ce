"""The allocation-free row_id_map entry point (moe_row_id_map_static_scratch).

It serves callers that may not allocate device memory when they build the
routing maps (a runtime that owns a fixed HBM budget, or a path where
cudaMalloc's implicit synchronisation is not allowed): its scratch is a
1 MiB device array inside the library. The GPU test calls it through the C
ABI several times in a row, on different problem sizes (up to the largest
the array accepts), and checks every output
against the workspace-based moe_row_id_map (integer outputs: bit-exact, the
tolerance used for all map tests). This file is collected last so that a
stop-at-first-failure run has already run every other test.
"""
from ctypes import byref, c_size_t

import numpy as np
import pytest
import torch

from oracle import moe_oracle as orc


def _lib():
    import moe_b200
    return moe_b200.load_library()


def _outputs(t, e, dev):
    return (torch.empty((e, t), dtype=torch.int64, device=dev),
            torch.empty((t, e), dtype=torch.int64, device=dev),
            torch.empty((e,), dtype=torch.int32, device=dev),
            torch.empty((1,), dtype=torch.int64, device=dev))


@pytest.mark.gpu
def test_static_scratch_matches_workspace_entry_point(cuda_dev):
    lib = _lib()
    stream = torch.cuda.current_stream(cuda_dev).cuda_stream
    g = torch.Generator().manual_seed(2024)
    # Calls in a row on the one shared array: each later call is smaller than
    # some earlier one, so stale counts left behind would show up in its maps.
    # (65408, 256) is the largest size the 1 MiB array accepts at E=256 (its
    # scratch ends exactly at the array's end); (64, 4096) takes the
    # single-block expert scan used for E > 2048.
    for t, e, align, p in ((16384, 256, 1, 8 / 256), (777, 300, 16, 0.05),
                           (65408, 256, 1, 8 / 256), (16384, 256, 128, 0.03),
                           (64, 4096, 1, 0.002)):
        rm = (torch.rand(t, e, generator=g) < p).to(cuda_dev)
        et_s, te_s, c_s, n_s = _outputs(t, e, cuda_dev)
        st = lib.moe_row_id_map_static_scratch(rm.data_ptr(), t, e, align, et_s.data_ptr(),
                                               te_s.data_ptr(), c_s.data_ptr(), n_s.data_ptr(),
                                               stream)
        assert st == 0, lib.moe_b200_last_error()
        et_w, te_w, c_w, n_w = _outputs(t, e, cuda_dev)
        nb = c_size_t(0)
        assert lib.moe_row_id_map_workspace_size(t, e, byref(nb)) == 0
        ws = torch.empty(nb.value, dtype=torch.uint8, device=cuda_dev)
        st = lib.moe_row_id_map(rm.data_ptr(), t, e, align, et_w.data_ptr(), te_w.data_ptr(),
                                c_w.data_ptr(), n_w.data_ptr(), ws.data_ptr(), nb.value, stream)
        assert st == 0, lib.moe_b200_last_error()
        torch.cuda.synchronize(cuda_dev)
        assert torch.equal(et_s, et_w) and torch.equal(te_s, te_w)
        assert torch.equal(c_s, c_w) and torch.equal(n_s, n_w)
        ref_et, ref_te, ref_c, ref_n = orc.row_id_map(rm.cpu().numpy(), align)
        np.testing.assert_array_equal(te_s.cpu().numpy(), ref_te)
        assert int(n_s.item()) == ref_n


def test_static_scratch_rejects_sizes_beyond_the_array():
    """Rejected before any device work, so this runs without a GPU."""
    lib = _lib()
    dummy = 256  # never dereferenced: the size check comes first
    for t in (1 << 17, 65409):  # far past the limit, and one token past it at E=256
        st = lib.moe_row_id_map_static_scratch(dummy, t, 256, 1, dummy, dummy, dummy, dummy,
                                               None)
        assert st == 1, t
        msg = lib.moe_b200_last_error()
        assert b"static array" in msg and b"moe_row_id_map" in msg
