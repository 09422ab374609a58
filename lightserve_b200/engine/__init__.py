"""CPU-side serving engine state: requests, KV-cache block tables and the
continuous-batching scheduler that feed the paged kernels."""
from .config import CacheConfig, SchedulerConfig
from .request import Request, RequestStatus, SamplingParams
from .block_manager import BlockManager, OutOfMemoryError
from .scheduler import ScheduledRequest, Scheduler, SchedulerOutput

__all__ = ["CacheConfig", "SchedulerConfig", "Request", "RequestStatus", "SamplingParams",
           "BlockManager", "OutOfMemoryError", "Scheduler", "SchedulerOutput", "ScheduledRequest"]
