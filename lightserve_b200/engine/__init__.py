"""CPU-side KV-cache bookkeeping (block tables) feeding the paged decode kernels."""
from .config import CacheConfig
from .request import Request, RequestStatus, SamplingParams
from .block_manager import BlockManager, OutOfMemoryError

__all__ = ["CacheConfig", "Request", "RequestStatus", "SamplingParams", "BlockManager",
           "OutOfMemoryError"]
