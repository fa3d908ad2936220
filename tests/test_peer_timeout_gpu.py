"""Failure detection of the cross-rank barrier, on one GPU and without a fault.

The barrier kernel is given two flag arrays in this GPU's memory, one standing
in for a peer that never arrives.  Its wait must run out after its 2 s bound,
record BS_ERR_DEVICE_TIMEOUT for the host, and leave the context usable; the
signal it sends to the silent "peer" must still have landed.
"""

from __future__ import annotations

import ctypes
import importlib
import time

import pytest
import torch

from conftest import PKG_NAME

pytestmark = pytest.mark.gpu


def test_barrier_wait_runs_out_and_reports():
    L = importlib.import_module(PKG_NAME + "._lib")
    pkg = importlib.import_module(PKG_NAME)
    lib = L.load()
    L.device_error_check()                      # start from a clean error word
    own = torch.zeros(2, dtype=torch.int64, device="cuda")
    peer = torch.zeros(2, dtype=torch.int64, device="cuda")   # nothing ever writes own[1]
    ptrs = (ctypes.c_void_p * 2)(own.data_ptr(), peer.data_ptr())
    t0 = time.time()
    L.check(lib.bs_peer_barrier(ptrs, 2, 0, 1, torch.cuda.current_stream().cuda_stream))
    with pytest.raises(L.BsError) as err:
        L.device_error_check()
    elapsed = time.time() - t0
    assert err.value.code == L.BS_ERR_DEVICE_TIMEOUT
    assert 1.5 < elapsed < 30, elapsed
    assert int(peer[0].item()) == 1             # our arrival reached the other rank's flags
    # the context is still usable
    x = torch.randn(4, 256, device="cuda").to(torch.bfloat16)
    y, s = pkg.act_quant(x, 128)
    torch.cuda.synchronize()
    assert y.shape == (4, 256) and torch.isfinite(s).all()
    L.device_error_check()
