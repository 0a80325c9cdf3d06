"""Host-side runtime of the zs B200 kernels: loader of libzs.so (the C ABI of
include/zs.h), build step, and small helpers shared by the drop-in modules."""
from . import _lib
from ._lib import ZsError, device_error, clear_device_error

__all__ = ["_lib", "ZsError", "device_error", "clear_device_error"]
