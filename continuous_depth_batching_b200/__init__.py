"""B200-native continuous depth batching (CDB) for looped language models.

Drop-in surface of ``looped_cdb.continuous_depth_batching``: build an engine with
``ContinuousDepthBatchingEngine.from_model(model, ContinuousDepthBatchingConfig(...))`` and call
``generate_batch``. Ouro and Huginn models are served. Compute runs in ``libcdb_b200.so`` (hand-written sm_100a kernels behind the C
ABI in ``include/cdb_b200.h``) plus cuBLAS GEMMs; there is no CPU path.
"""

from .config import ContinuousDepthBatchingConfig
from .engine import (
    CacheFullError,
    ContinuousDepthBatchingEngine,
    ContinuousDepthBatchingStats,
    GenerationOutput,
    RequestStatus,
)
from .huginn import HuginnForCausalLM, HuginnShape, random_huginn_state_dict
from .ouro import OuroForCausalLM, OuroShape, random_ouro_state_dict

__all__ = [
    "CacheFullError",
    "ContinuousDepthBatchingConfig",
    "ContinuousDepthBatchingEngine",
    "ContinuousDepthBatchingStats",
    "GenerationOutput",
    "HuginnForCausalLM",
    "HuginnShape",
    "OuroForCausalLM",
    "OuroShape",
    "RequestStatus",
    "random_huginn_state_dict",
    "random_ouro_state_dict",
]
