"""lightserve_b200: B200-native (sm_100a) attention hot path of lightserve.

Operators (drop-ins for lightserve's ``kernels/`` call sites) live in
``lightserve_b200.kernels``; the paged-KV decode driver in
``lightserve_b200.model``; block-table bookkeeping in ``lightserve_b200.engine``.
All compute goes through liblightserve_b200.so (include/lightserve_b200.h).
"""
__version__ = "0.1.0"
