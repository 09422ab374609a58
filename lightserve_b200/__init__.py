"""lightserve_b200: B200-native (sm_100a) attention hot path of lightserve.

Operators (drop-ins for lightserve's ``kernels/`` call sites) live in
``lightserve_b200.kernels``; the paged-KV decode driver in
``lightserve_b200.model``; block-table bookkeeping in ``lightserve_b200.engine``.
All compute goes through liblightserve_b200.so (include/lightserve_b200.h).
"""
__version__ = "0.1.0"


from ._lib import DeviceWaitError  # noqa: E402


def check_device_errors(reset: bool = True) -> None:
    """Raises if a kernel of the library gave up on a bounded on-chip wait
    (see ``lightserve_b200._lib.check_device_errors``)."""
    from ._lib import check_device_errors as _check

    _check(reset)
