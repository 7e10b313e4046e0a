"""Failure detection on the GPU without a fault: a bounded device wait that runs out reports
MF_DEVICE_TIMEOUT through the sticky status and leaves the context usable."""
import ctypes
import time

import numpy as np
import pytest

from manifesto_b200._abi import call
from manifesto_b200.backend import DeviceBuffer, PinnedBuffer, Stream
from manifesto_b200.errors import DeviceStickyError
from oracle.ref import BF16, F32

from .gpu_util import convert, to_device

pytestmark = pytest.mark.gpu

MF_DEVICE_TIMEOUT = 0x7100


def status():
    code = ctypes.c_int(0)
    try:
        call("mf_device_status", ctypes.byref(code))
    except DeviceStickyError:
        return code.value
    return code.value


def test_wait_on_a_flag_nothing_sets_times_out(backend, ref):
    flag = to_device(np.zeros(1, np.int32))
    t0 = time.perf_counter()
    call("mf_wait_flag", flag.ptr, 1, 20000, None)   # ~20000 polls of ~0.3 us
    assert status() == MF_DEVICE_TIMEOUT            # read and cleared
    assert time.perf_counter() - t0 < 30
    assert status() == 0
    # the context is still usable and the next status is clean
    x = np.arange(4096, dtype=np.float32) * 0.25
    got = convert(x, F32, BF16, 4096)
    assert np.array_equal(got, ref.convert(x, F32, BF16))
    assert status() == 0
    flag.free()


def test_wait_returns_when_the_flag_is_set(backend):
    flag = to_device(np.array([7], np.int32))
    call("mf_wait_flag", flag.ptr, 7, 1 << 20, None)  # already set: returns on the first poll (budget ~0.3 s)
    assert status() == 0
    # set by a host-to-device copy on another stream while the wait is running
    flag2 = to_device(np.zeros(1, np.int32))
    host = PinnedBuffer(4)
    host.array.view(np.int32)[0] = 3
    waiter, setter = Stream(), Stream()
    call("mf_wait_flag", flag2.ptr, 3, 1 << 22, waiter.handle)  # budget ~1 s, never reached
    call("mf_memcpy_h2d_async", flag2.ptr, host.ptr, 4, setter.handle)
    waiter.sync()
    setter.sync()
    assert status() == 0
    for b in (flag, flag2):
        b.free()
    host.free()
    waiter.close()
    setter.close()


def test_wait_flag_rejects_bad_arguments(backend):
    from manifesto_b200.errors import InvalidArgument
    with pytest.raises(InvalidArgument, match="flag is NULL"):
        call("mf_wait_flag", None, 0, 1, None)
    buf = DeviceBuffer(16)
    with pytest.raises(InvalidArgument, match="not 4-byte aligned"):
        call("mf_wait_flag", buf.ptr + 2, 0, 1, None)
    with pytest.raises(InvalidArgument, match="negative poll budget"):
        call("mf_wait_flag", buf.ptr, 0, -1, None)
    buf.free()
