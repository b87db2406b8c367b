"""ds_copy_ranges argument checks run on the host, before any CUDA call."""
from __future__ import annotations

import ctypes
import threading

import pytest

from deepseeker import _abi, _build


@pytest.fixture(scope="module")
def lib():
    _build.build(verbose=False)
    return _abi.lib()


def ranges(*triples):
    n = len(triples)
    return (n, (ctypes.c_void_p * max(n, 1))(*[t[0] for t in triples]),
            (ctypes.c_void_p * max(n, 1))(*[t[1] for t in triples]),
            (ctypes.c_size_t * max(n, 1))(*[t[2] for t in triples]))


def _checks():
    # (addresses are never dereferenced: every case fails its checks first)
    for bad in (ranges(), ranges(*[(4096, 8192, 16)] * 5),          # 0 or 5 ranges
                ranges((4096 + 8, 8192, 16)), ranges((4096, 8192 + 4, 16)),   # misaligned
                ranges((4096, 8192, 24)), ranges((0, 8192, 16))):   # size not a multiple of 16, null
        with pytest.raises(ValueError):
            _abi.call("ds_copy_ranges", *bad, None)
    d = ctypes.c_void_p(0)
    with pytest.raises(ValueError):
        _abi.call("ds_host_device_pointer", None, ctypes.byref(d))


def test_copy_ranges_checks_need_no_gpu(lib):
    # in a thread of its own: the library's last-error string is per thread,
    # and other tests expect this thread's to be empty
    errors = []

    def run():
        try:
            _checks()
        except BaseException as e:  # noqa: BLE001 (re-raised below)
            errors.append(e)

    t = threading.Thread(target=run)
    t.start()
    t.join()
    if errors:
        raise errors[0]
