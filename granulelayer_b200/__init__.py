"""B200-native (sm_100a) sparse-pooling layer: a drop-in for the reference
``sparse_pooling`` package's Mode-A fp32 hot path.

About 10^8 logical neurons each compute ``act(b + sum_{k<8} w_k x[idx_k])``
and are pooled into contiguous groups without materialising the [B, H]
hidden tensor; backward gives dX, dW, db; ``FusedAdamW`` applies the
optimizer in one pass.  All GPU work runs in the in-tree library
``_lib/libgranule_b200.so`` through the C ABI of ``include/granule_b200.h``.
"""
from .config import LevelSpec, PhysicalPlan, PoolingConfig
from .layer import SparsePoolingLayer
from .layout import SparseLayout, init_parameters
from .optim import FusedAdamW

__all__ = ["SparsePoolingLayer", "PoolingConfig", "LevelSpec", "PhysicalPlan", "SparseLayout", "init_parameters",
           "FusedAdamW"]
