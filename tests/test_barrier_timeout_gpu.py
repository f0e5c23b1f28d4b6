"""The device barrier's bounded wait, made to run out on one GPU.

``mxfp4_peer_barrier_timed`` with world = 2 on a single device: rank 0's own
flag array is a local buffer, and "rank 1"'s flag array is a second local
buffer that no kernel ever signals.  The barrier stores its signals, waits
10 ms for the missing one, records MXFP4_ERR_TIMEOUT in the device status word
and returns: no fault, no hang, the context stays usable.  The collective
reset (``mxfp4_peer_barrier_reset``) then zeroes the flags and the counter,
after which a barrier completes with status 0.
"""

import ctypes
import time

import pytest
import torch

from _paths import soft_module

pytestmark = pytest.mark.gpu
soft = soft_module()
ERR_TIMEOUT = 4


def _ptrs(*tensors):
    arr = (ctypes.c_void_p * len(tensors))(*[t.data_ptr() for t in tensors])
    return ctypes.cast(arr, ctypes.POINTER(ctypes.c_void_p))


def test_barrier_wait_runs_out_and_reset_recovers():
    lib = soft._load_library()
    soft.device_status(0)  # start from a clean status word
    mine = torch.zeros(8, dtype=torch.int32, device="cuda")
    silent_peer = torch.zeros(8, dtype=torch.int32, device="cuda")  # nobody signals rank 0 here
    counter = torch.zeros(1, dtype=torch.int32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    t0 = time.perf_counter()
    rc = lib.mxfp4_peer_barrier_timed(_ptrs(mine, silent_peer), 0, 2, ctypes.c_void_p(counter.data_ptr()), 10_000,
                                      ctypes.c_void_p(stream))
    assert rc == 0, lib.mxfp4_last_error()
    torch.cuda.synchronize()
    waited = time.perf_counter() - t0
    assert soft.device_status(0) == ERR_TIMEOUT  # reads and clears the word
    assert 0.005 < waited < 5.0, waited
    # the barrier signalled both ranks with epoch 1 before it waited
    assert counter.item() == 1 and mine[0].item() == 1 and silent_peer[0].item() == 1
    # reset this rank's flags and counter (the local step of the collective reset)
    rc = lib.mxfp4_peer_barrier_reset(ctypes.c_void_p(mine.data_ptr()), 2, ctypes.c_void_p(counter.data_ptr()),
                                      ctypes.c_void_p(stream))
    assert rc == 0
    torch.cuda.synchronize()
    assert counter.item() == 0 and int(mine[:2].abs().sum()) == 0
    # a barrier whose every signal arrives (world 1) completes with status 0
    rc = lib.mxfp4_peer_barrier_timed(_ptrs(mine), 0, 1, ctypes.c_void_p(counter.data_ptr()), 10_000,
                                      ctypes.c_void_p(stream))
    assert rc == 0
    torch.cuda.synchronize()
    assert soft.device_status(0) == 0 and counter.item() == 1
