"""B200-native continuous depth batching (CDB) for looped language models.

Drop-in surface of ``looped_cdb.continuous_depth_batching``: build an engine with
``ContinuousDepthBatchingEngine.from_model(model, ContinuousDepthBatchingConfig(...))`` and call
``generate_batch``. Ouro and Huginn models are served. ``ContinuousBatchingEngine`` is the
full-depth continuous-batching baseline on the same kernels. Compute runs in ``libcdb_b200.so`` (hand-written sm_100a kernels behind the C
ABI in ``include/cdb_b200.h``) plus cuBLAS GEMMs; there is no CPU path.
"""

from .cb_engine import ContinuousBatchingConfig, ContinuousBatchingEngine, ContinuousBatchingStats, DecodeStepTiming
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
    "ContinuousBatchingConfig",
    "ContinuousBatchingEngine",
    "ContinuousBatchingStats",
    "ContinuousDepthBatchingConfig",
    "ContinuousDepthBatchingEngine",
    "ContinuousDepthBatchingStats",
    "DecodeStepTiming",
    "GenerationOutput",
    "HuginnForCausalLM",
    "HuginnShape",
    "OuroForCausalLM",
    "OuroShape",
    "RequestStatus",
    "random_huginn_state_dict",
    "random_ouro_state_dict",
]
