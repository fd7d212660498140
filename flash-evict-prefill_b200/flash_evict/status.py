"""Errors that kernels report after their call has returned.

Every call into the native library is asynchronous: it validates, launches
and returns before the kernels run.  A kernel that gives up on a device-side
wait (the watchdog limit, 2 s by default) cannot fail the call that launched
it, so it records a status code in two places:

* a mapped pinned host word per device, which every later call on that
  device reads on entry (plain host memory, no synchronization): the code
  becomes that call's error -- a RuntimeError naming the device watchdog
  timeout -- and is cleared, and that call launches nothing;
* the device status word, which `check_status` reads after synchronizing
  the device.

Outputs of the call whose kernel gave up hold NaN where the kernel could
mark them (attention rows, their statistics, importance, SnapKV scores).
"""
import torch

from . import _lib

__all__ = ["check_status"]


def check_status(device=None):
    """Synchronize `device` (default: the current CUDA device) and raise
    RuntimeError if any kernel of this library reported a failure there since
    the last check (a device watchdog timeout, or a gather index out of range).
    The record is cleared, so a second call returns normally.  A failure that
    an earlier call already raised is reported here again: the device record
    is kept until this check (or `fe_device_status`) clears it."""
    if device is None:
        dev = torch.cuda.current_device()
    else:
        d = torch.device(device) if not isinstance(device, int) else torch.device("cuda", device)
        dev = d.index if d.index is not None else torch.cuda.current_device()
    code = _lib.device_status(dev, clear=True)
    if code != _lib.STATUS_OK:
        raise RuntimeError(f"flash_evict: a kernel on cuda:{dev} reported "
                           f"{_lib.status_name(code)} (status {code})")
